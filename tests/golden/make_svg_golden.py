"""Generate golden SVG-EAR value-error scores by running the REFERENCE Triton
kernel on the CPU through Triton's interpreter.

Run in a container that has the reference checkout (it is never read at test
time):

    python tests/golden/make_svg_golden.py /path/to/SparsePR

The reference's ``_svg_ear_value_error_kernel``
(``src/sparsepr/kernels/triton/svg_ear.py:95-193``) is launched exactly as its
wrapper ``svg_ear_value_error_scores_triton`` (453-531) launches it for the
route (no Jensen term, ``n8_v6.py:984-998``), with ``TRITON_INTERPRET=1`` so it
executes on CPU tensors; the wrapper itself is bypassed only because it
refuses non-CUDA tensors.  Output: ``tests/golden/svg_ear_value_scores.pt``.
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    import triton
    from sparsepr.kernels.triton.svg_ear import _svg_ear_value_error_kernel

    cases = []
    for seed, (h, cq, ck, n, qscale) in enumerate([(2, 10, 12, 150, 1.0), (1, 20, 9, 120, 3.0)]):
        g = torch.Generator().manual_seed(100 + seed)
        d = 128
        q = torch.randn(h, cq, d, generator=g) * qscale
        ks = torch.randn(h, n, d, generator=g).bfloat16()
        vs = torch.randn(h, n, d, generator=g).bfloat16()
        lab = torch.randint(0, ck - 2, (h, n), generator=g)  # two empty clusters at the end
        sizes = torch.zeros(h, ck, dtype=torch.long).scatter_add_(1, lab, torch.ones_like(lab)).int()
        kc = torch.randn(h, ck, d, generator=g)
        vc = torch.randn(h, ck, d, generator=g)
        off = torch.cat([torch.zeros(h, 1, dtype=torch.int32), sizes.cumsum(1).int()], 1).contiguous()
        scores = torch.empty(h, cq, ck)
        grid = (triton.cdiv(cq, 16), ck, h)
        _svg_ear_value_error_kernel[grid](
            q, ks, vs, kc, vc, kc, off, scores, Q_CLUSTERS=cq, K_CLUSTERS=ck, TOKENS=n, SORTED_HEAD_STRIDE=n,
            DIM=d, GQA_GROUP=1, JENSEN_VAR_CAP=0.0, USE_JENSEN=False, BLOCK_Q=16, BLOCK_N=32)
        cases.append(dict(q_centroids=q, k_sorted=ks, v_sorted=vs, k_centroids=kc, v_centroids=vc,
                          k_sizes=sizes, scores=scores))
    torch.save(cases, os.path.join(HERE, "svg_ear_value_scores.pt"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_svg_golden.py /path/to/SparsePR")
    main(sys.argv[1])
