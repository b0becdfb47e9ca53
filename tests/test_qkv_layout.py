"""Wan producer step (RMSNorm + RoPE + BHLD layout): oracle known answers on
CPU, and the CUDA kernel (through the C ABI) against the oracle on the GPU."""

import math

import pytest
import torch

import oracle


def test_oracle_known_answer():
    # One token, 2 heads of head_dim 2, unit inputs and weights, eps 0: the
    # norm is exactly 1, so each head's pair (1, 1) is rotated by its angle.
    q = torch.ones(1, 1, 4)
    w = torch.ones(4)
    th = 0.3
    fr = torch.tensor([[math.cos(th)]])
    fi = torch.tensor([[math.sin(th)]])
    qo, ko, vo = oracle.wan_qkv_norm_rope_layout(q, 2 * q, 3 * q, w, w, fr, fi, heads=2, epsilon=0.0)
    want = torch.tensor([math.cos(th) - math.sin(th), math.sin(th) + math.cos(th)])
    assert qo.shape == (1, 2, 1, 2)
    torch.testing.assert_close(qo[0, :, 0], want.expand(2, 2))
    torch.testing.assert_close(ko, qo)  # the norm removes the factor 2
    assert torch.equal(vo, torch.full((1, 2, 1, 2), 3.0))


def test_oracle_keeps_model_dtype():
    # bf16 in, bf16 out; the weight scales each channel of the normalised row.
    x = torch.tensor([[[1.0, 1.0 + 2 ** -10]]]).bfloat16()  # second value rounds to 1.0 in bf16 already
    w = torch.tensor([1.0, 1.0 + 2 ** -7]).bfloat16()
    qo, _, _ = oracle.wan_qkv_norm_rope_layout(x, x, x, w, w, torch.ones(1, 1), torch.zeros(1, 1), heads=1,
                                               epsilon=0.0)
    assert qo.dtype == torch.bfloat16
    assert qo[0, 0, 0].tolist() == [1.0, 1.0 + 2 ** -7]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hd", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 128)])
def test_kernel_matches_oracle(cuda, dtype, hd):
    from sparsepr_b200 import kernels as K

    g = torch.Generator().manual_seed(hd)
    b, l, h = 2, 300, 5
    c = h * hd
    q, k, v = (torch.randn(b, l, c, generator=g).to(dtype) for _ in range(3))
    k = k * 3
    qw, kw = (1 + 0.1 * torch.randn(c, generator=g)).to(dtype), (1 + 0.1 * torch.randn(c, generator=g)).to(dtype)
    ang = torch.rand(l, hd // 2, generator=g) * 6.3
    fr, fi = ang.cos(), ang.sin()
    ref = oracle.wan_qkv_norm_rope_layout(q, k, v, qw, kw, fr, fi, heads=h, epsilon=1e-6)
    got = K.wan_qkv_norm_rope_layout(*(t.to(cuda) for t in (q, k, v, qw, kw, fr, fi)), heads=h, epsilon=1e-6)
    assert torch.equal(got[2].cpu(), ref[2])  # V: layout only
    for o, r in zip(got[:2], ref[:2]):
        o = o.cpu()
        assert o.shape == (b, h, l, hd) and o.dtype == dtype
        # The row norm's summation order and rsqrt differ from the oracle in the
        # last fp32 bits, which can move a value across one rounding boundary.
        same = (o == r).float().mean().item()
        assert same > (0.99 if dtype != torch.float32 else 0.0), same
        eps = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 1e-6}[dtype]
        torch.testing.assert_close(o.float(), r.float(), rtol=2 * eps, atol=2 * eps)


@pytest.mark.gpu
def test_kernel_rejects_bad_shapes(cuda):
    from sparsepr_b200 import kernels as K

    q = torch.zeros(1, 4, 12, dtype=torch.bfloat16, device=cuda)  # head_dim 6 is not a multiple of 8
    w = torch.ones(12, dtype=torch.bfloat16, device=cuda)
    f = torch.ones(4, 3, device=cuda)
    with pytest.raises(RuntimeError):
        K.wan_qkv_norm_rope_layout(q, q, q, w, w, f, f, heads=2, epsilon=1e-6)


def test_install_patch_replaces_the_reference_entry_points():
    import types

    from sparsepr_b200 import attention as A
    from sparsepr_b200 import kernels as K

    adapter = types.SimpleNamespace(_sparse_n8_attention_bhld="ref attn", _make_n8_core="ref core")
    ext = types.SimpleNamespace(wan_qkv_norm_rope_layout="ref qkv")
    prev = A.install_wan22_ti2v_sparse_patch(module=adapter, extension_module=ext)
    assert prev == ("ref attn", "ref core")
    assert adapter._sparse_n8_attention_bhld is A.sparse_n8_attention_bhld
    assert adapter._make_n8_core is A.make_n8_core
    assert ext.wan_qkv_norm_rope_layout is K.wan_qkv_norm_rope_layout


def test_install_hunyuan_patch_replaces_the_processor_method():
    from sparsepr_b200 import attention as A

    class Processor:
        def _sparse_attention(self, query, key, value):
            return "reference"

    old = Processor._sparse_attention
    prev = A.install_hunyuan_sparse_patch(Processor)
    assert prev is old and Processor._sparse_attention is not old


def _reference_src():
    """The reference checkout's src/ next to this repository, when present (it is
    only in the build container, never on a GPU box)."""
    import os

    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = os.path.join(os.path.dirname(here), "reference", "src")
    return src if os.path.isdir(os.path.join(src, "sparsepr", "adapters")) else None


def test_install_into_the_real_reference_adapter():
    """The patch installed into the reference's own sparsepr.adapters.wan22: its
    _sparse_n8_attention (wan22.py:1926-1942) then runs this build's body
    (BLHD -> BHLD conversion by the reference, routing here), and its core
    factory builds this build's N8V6Core.  On the CPU the build's routing
    refuses the call, which proves the call reached it."""
    import importlib
    import sys
    import types

    src = _reference_src()
    if src is None:
        pytest.skip("reference sources not present")
    sys.path.insert(0, src)
    try:
        wan22 = importlib.import_module("sparsepr.adapters.wan22")
    except Exception as e:  # an optional dependency of the adapter module is missing
        pytest.skip(f"reference adapter does not import here: {e!r}")
    finally:
        sys.path.remove(src)
    from sparsepr_b200 import N8V6Core
    from sparsepr_b200 import attention as A

    prev = A.install_wan22_ti2v_sparse_patch(module=wan22)
    try:
        assert wan22._sparse_n8_attention_bhld is A.sparse_n8_attention_bhld
        assert isinstance(wan22._make_n8_core(), N8V6Core)
        attn = types.SimpleNamespace()
        q = torch.randn(1, 64, 2, 128)  # [B, L, H, D] as the Wan attention passes it
        with pytest.raises(RuntimeError, match="sparsepr_b200 N8-V6 routing runs on CUDA tensors only"):
            wan22._sparse_n8_attention(attn, q, q, q, None)
        assert isinstance(attn._n8_cores[0], N8V6Core)  # the branch-local core cache of wan22.py:1551-1566
    finally:
        wan22._sparse_n8_attention_bhld, wan22._make_n8_core = prev


def _wan_fixture():
    import os
    import sys

    golden = os.path.join(os.path.dirname(__file__), "golden")
    sys.path.insert(0, golden)
    try:
        from make_wan_qkv_golden import cases, inputs
    finally:
        sys.path.remove(golden)
    fx = torch.load(os.path.join(golden, "wan_qkv_layout_ref.pt"))
    return cases(), inputs, fx["cases"]


def _check_against_reference(got, want, dtype):
    assert torch.equal(got[2], want[2])  # V: layout only
    for o, r in zip(got[:2], want[:2]):
        assert o.shape == r.shape and o.dtype == r.dtype
        # The reference is built with fast math (approximate rsqrt); values may
        # sit one rounding step apart.
        same = (o == r).float().mean().item()
        assert same > (0.98 if dtype != torch.float32 else 0.0), same
        eps = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 1e-6}[dtype]
        torch.testing.assert_close(o.float(), r.float(), rtol=2 * eps, atol=2 * eps)


def test_oracle_matches_reference_kernel_outputs():
    """The oracle restatement against the reference's own CUDA kernel's outputs
    (tests/golden/wan_qkv_layout_ref.pt, make_wan_qkv_golden.py)."""
    specs, make_inputs, recs = _wan_fixture()
    for (dtype, b, l, h, hd), rec in zip(specs, recs):
        args = make_inputs(dtype, b, l, h, hd, rec["seed"])
        got = oracle.wan_qkv_norm_rope_layout(*args, heads=h, epsilon=rec["epsilon"])
        _check_against_reference(got, rec["outputs"], dtype)


@pytest.mark.gpu
def test_kernel_matches_reference_kernel_outputs(cuda):
    from sparsepr_b200 import kernels as K

    specs, make_inputs, recs = _wan_fixture()
    for (dtype, b, l, h, hd), rec in zip(specs, recs):
        args = make_inputs(dtype, b, l, h, hd, rec["seed"])
        got = K.wan_qkv_norm_rope_layout(*(t.to(cuda) for t in args), heads=h, epsilon=rec["epsilon"])
        _check_against_reference([t.cpu() for t in got], rec["outputs"], dtype)
