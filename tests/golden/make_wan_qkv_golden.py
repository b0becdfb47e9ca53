"""Wan Q/K/V producer fixture from the REFERENCE's own CUDA kernel.

    python -m oracle.build_ref                     # in the container with the reference checkout
    python tests/golden/make_wan_qkv_golden.py     # on a GPU (the prebuilt module travels)

Runs ``n8_kernels.wan_qkv_norm_rope_layout`` (``src/sparsepr/kernels/n8_ext/
csrc/n8_ops.cu:16-105, 357-411``, built by ``oracle/build_ref.py`` with the
reference's own compiler flags) on seeded inputs in bf16, fp16 and fp32 and
writes inputs and outputs to ``tests/golden/wan_qkv_layout_ref.pt`` (or to the
path given as the first argument).
"""

from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def cases():
    """(dtype, batch, tokens, heads, head_dim) of the fixture."""
    return [(torch.bfloat16, 1, 96, 4, 128), (torch.float16, 2, 40, 3, 64), (torch.float32, 1, 64, 2, 128)]


def inputs(dtype, b, l, h, hd, seed):
    g = torch.Generator().manual_seed(seed)
    c = h * hd
    q, k, v = (torch.randn(b, l, c, generator=g).to(dtype) for _ in range(3))
    k = (k.float() * 3).to(dtype)
    qw = (1 + 0.1 * torch.randn(c, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(c, generator=g)).to(dtype)
    ang = torch.rand(l, hd // 2, generator=g) * 6.3
    return q, k, v, qw, kw, ang.cos().contiguous(), ang.sin().contiguous()


def main(out_path: str) -> None:
    sys.path.insert(0, REPO)
    from oracle.build_ref import load_reference_kernels

    ref = load_reference_kernels()
    dev = torch.device("cuda")
    records = []
    for i, (dtype, b, l, h, hd) in enumerate(cases()):
        args = inputs(dtype, b, l, h, hd, seed=100 + i)
        outs = ref.wan_qkv_norm_rope_layout(*(t.to(dev) for t in args), h, 1e-6)
        torch.cuda.synchronize()
        records.append({"dtype": str(dtype), "shape": (b, l, h, hd), "seed": 100 + i, "epsilon": 1e-6,
                        "outputs": [o.cpu() for o in outs]})
    torch.save({"cases": records}, out_path)
    print("wrote", out_path, len(records), "cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "wan_qkv_layout_ref.pt"))
