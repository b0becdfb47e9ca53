"""sparsepr_b200: B200-native (sm_100a) SparsePR sparse-attention hot path.

Public API:

* :class:`N8V6Config`, :class:`N8V6Core`, :class:`N8V6Route` — the routing +
  repair core (drop-in for ``sparsepr.models.common.n8_v6``).
* :func:`sparse_attention` — the adapter-facing attention call.
* :class:`RouteCache` — route reuse across steps and CFG branches.
* :func:`batch_kmeans_Euclid`, :class:`FlashKMeans` — standalone batched k-means.
* :func:`check_status` — raise if a device-side bounded wait of the last layer gave up.
* :mod:`sparsepr_b200.kernels` — tensor wrappers over the C ABI.
"""

from .n8_v6 import N8V6Config, N8V6Core, N8V6Route  # noqa: F401
from .attention import (  # noqa: F401
    Wan22TI2VSparseConfig,
    hunyuan_sparse_attention,
    install_hunyuan_sparse_patch,
    install_wan22_ti2v_sparse_patch,
    kept_flops,
    make_n8_core,
    sparse_attention,
)
from .route_cache import RouteCache, RouteReuseConfig, route_action  # noqa: F401
from .kmeans import FlashKMeans, batch_kmeans_Euclid  # noqa: F401
from .kernels import wan_qkv_norm_rope_layout  # noqa: F401


def check_status(device=None) -> None:
    """Wait for the status words of the last SparsePR layer on ``device`` (default:
    the current CUDA device) and raise ``RuntimeError`` if a device-side bounded
    wait gave up during it."""
    import torch

    from .kernels import raise_device_status

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    raise_device_status(dev, wait=True)

__version__ = "0.1.0"
