"""Device status words reach the host: the bounded device wait gives up and
reports (no trap, the context stays usable), and a non-zero status word of a
layer raises RuntimeError on the product path."""

import pytest
import torch

from sparsepr_b200 import _lib, check_status
from sparsepr_b200 import kernels as K

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(cuda):
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("spr_selftest_bounded_wait", err.data_ptr(), 7, 1_000_000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 7
    # The context is still usable after the wait gave up.
    x = torch.ones(1024, device=cuda)
    assert float(x.sum().item()) == 1024.0


def test_layer_status_words_raise_on_next_call(cuda):
    from sparsepr_b200 import N8V6Config, N8V6Core, sparse_attention
    from sparsepr_b200.synthetic import synthetic_qkv

    cfg = N8V6Config(num_q_centroids=16, num_k_centroids=24, target_density=0.3, kmeans_iter_init=3,
                     probe_rows=16, repair_rank=16, selector_policy="attention_mass",
                     role_kv_matmul_precision="highest", kmeans_precision="fp32")
    q, k, v = (t.to(cuda) for t in synthetic_qkv(2, 128, (4, 8, 8), dtype=torch.bfloat16))
    sparse_attention(q, k, v, N8V6Core(cfg))
    check_status(cuda)  # a clean layer: all words zero
    # Fake a wait that gave up inside the k-means of this layer (host-side injection).
    ws = K._WS[(cuda.type, cuda.index, "", "kmeans")]
    ws[:4].view(torch.int32).fill_(3)
    K.collect_status(cuda)
    with pytest.raises(RuntimeError, match="kmeans"):
        check_status(cuda)
    ws[:4].view(torch.int32).zero_()
    K.collect_status(cuda)
    check_status(cuda)
    # The next layer call raises when the previous layer's snapshot is bad.
    ws[:4].view(torch.int32).fill_(3)
    K.collect_status(cuda)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device status"):
        sparse_attention(q, k, v, N8V6Core(cfg))
    ws[:4].view(torch.int32).zero_()
