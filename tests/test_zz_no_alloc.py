"""The no-allocation attention entry point, through the C ABI.

Some callers cannot allocate device memory (a host that owns all of HBM
through its own pool, or a loop that must not call cudaMalloc and has no
buffer to lend), so ``spr_block_sparse_attn_noalloc`` keeps its scratch in a
fixed library-owned device array.  Two calls in a row, on different cluster
layouts, must agree with the workspace entry point ``spr_block_sparse_attn``.
This file is collected last on purpose.
"""

import pytest
import torch

from sparsepr_b200 import _lib
from sparsepr_b200 import kernels as K

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


def _layout(g, bh, n, cq, ck, density):
    def sizes_for(c):
        lab = torch.randint(0, c, (bh, n), generator=g)
        return torch.zeros(bh, c, dtype=torch.long).scatter_add_(1, lab, torch.ones_like(lab))

    qs, ks = sizes_for(cq), sizes_for(ck)
    mask = torch.rand(bh, cq, ck, generator=g) < density
    ids = torch.full((bh, cq, ck), -1, dtype=torch.int32)
    cnt = mask.sum(-1).to(torch.int32)
    for b in range(bh):
        for c in range(cq):
            sel = torch.nonzero(mask[b, c]).flatten()
            ids[b, c, : sel.numel()] = sel.to(torch.int32)
    off = lambda s: torch.cat((torch.zeros(bh, 1, dtype=torch.long), s.cumsum(1)), 1).to(torch.int32)  # noqa: E731
    return off(qs), off(ks), ids, cnt


def _noalloc(q, k, v, q_off, k_off, ids, cnt, q_order=None):
    bh, nq, d = q.shape
    out = torch.empty_like(q)
    _lib.call("spr_block_sparse_attn_noalloc", q.data_ptr(), k.data_ptr(), v.data_ptr(), q_off.data_ptr(),
              k_off.data_ptr(), ids.data_ptr(), cnt.data_ptr(), bh, nq, k.shape[1], d, q_off.shape[1] - 1,
              k_off.shape[1] - 1, None if q_order is None else q_order.data_ptr(), out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return out


def _noalloc_status():
    import ctypes

    code = ctypes.c_int(-1)
    _lib.call("spr_block_sparse_attn_noalloc_status", ctypes.addressof(code))
    return code.value


@pytest.mark.parametrize("fused_store", [False, True])
def test_noalloc_matches_workspace_entry_twice(cuda, fused_store):
    for call, (seed, n, cq, ck) in enumerate([(1, 2000, 13, 50), (2, 1300, 7, 31)]):
        g = torch.Generator().manual_seed(seed)
        bh = 3
        q, k, v = (torch.randn(bh, n, 128, generator=g).to(torch.bfloat16).to(cuda) for _ in range(3))
        q_off, k_off, ids, cnt = (t.to(cuda) for t in _layout(g, bh, n, cq, ck, 0.3))
        order = None
        if fused_store:
            order = torch.stack([torch.randperm(n, generator=g) for _ in range(bh)]).to(torch.int32).to(cuda)
        ref = K.block_sparse_attention(q, k, v, q_off, k_off, ids, cnt, q_order=order)
        got = _noalloc(q, k, v, q_off, k_off, ids, cnt, order)
        torch.cuda.synchronize()
        assert _noalloc_status() == 0, call  # no bounded device wait gave up
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= ATOL, (call, err)
        for h in range(bh):
            a, b = got[h].float().flatten(), ref[h].float().flatten()
            if b.norm() > 0:
                assert torch.nn.functional.cosine_similarity(a, b, dim=0).item() >= COS


def test_noalloc_rejects_oversized_problems(cuda):
    # 400 problems x (200 + 1) tile-table entries > the fixed 65,536: rejected before any launch.
    with pytest.raises(RuntimeError, match="SPR_ERR_SHAPE.*fixed scratch"):
        _lib.call("spr_block_sparse_attn_noalloc", 16, 16, 16, None, None, None, None, 400, 1000, 1000, 128, 200,
                  1000, None, 16, None)
