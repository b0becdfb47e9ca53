"""Random-init HunyuanVideo-architecture DiT: the caller of the Hunyuan SparsePR boundary.

A synthetic denoising-step workload around :func:`sparsepr_b200.attention.hunyuan_sparse_attention`
(the reference's ``HunyuanVideoN8Processor._sparse_attention``,
``src/sparsepr/adapters/hunyuanvideo.py:160-239``), with the block structure of the
public HunyuanVideo description: patch embedding of the 16-channel latent (patch
1x2x2), a timestep / pooled-text / guidance vector, ``double_blocks`` dual-stream
blocks (separate video and text weights, joint attention) and ``single_blocks``
single-stream blocks (one fused linear for QKV and the MLP input), adaLN
modulation from the vector, per-head RMS normalisation of Q and K, 3-D rotary
position embedding on video tokens, and a modulated output projection.  The
text token refiner is replaced by one linear projection.  Weights are random;
nothing here is trained or loaded.

Attention in every block is SparsePR on the video tokens with the text context
appended (video rows attend video clusters and the prompt; text rows as the
boundary defines).  With a process group of W ranks the video tokens are
sequence-sharded: the dense layers run on N/W video tokens per rank (text
replicated), and around each attention call an all-to-all regroups Q/K/V into
head shards (H/W heads, all tokens) and returns the output (Ulysses); the text
rows' output heads are all-gathered.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

__all__ = ["HunyuanDiTConfig", "HunyuanDiT", "JointAttention", "SparsePRBlocks", "rope_3d"]


@dataclass
class HunyuanDiTConfig:
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    mlp_ratio: float = 4.0
    double_blocks: int = 20
    single_blocks: int = 40
    in_channels: int = 16
    patch: tuple = (1, 2, 2)
    text_dim: int = 4096
    vec_dim: int = 768
    rope_axes: tuple = (16, 56, 56)
    rope_theta: float = 256.0

    def validate(self) -> None:
        if self.heads * self.head_dim != self.hidden:
            raise ValueError(f"heads x head_dim = {self.heads * self.head_dim} must equal hidden {self.hidden}.")
        if sum(self.rope_axes) != self.head_dim or any(a % 2 for a in self.rope_axes):
            raise ValueError(f"rope axes {self.rope_axes} must be even and sum to head_dim {self.head_dim}.")


def rope_3d(grid, positions, axes, theta, device):
    """cos/sin [n, head_dim/2] of 3-D rotary embedding for token indices ``positions``
    (row-major over the (t, h, w) ``grid``); channel pairs (2i, 2i+1) rotate together,
    the first ``axes[0]`` channels by t, the next ``axes[1]`` by h, the last by w."""
    t_, h_, w_ = grid
    pos = positions.to(device)
    coords = (pos // (h_ * w_), (pos // w_) % h_, pos % w_)
    angles = []
    for c, dim in zip(coords, axes):
        inv = theta ** (-torch.arange(0, dim, 2, device=device, dtype=torch.float64) / dim)
        angles.append(c.double()[:, None] * inv[None, :])
    ang = torch.cat(angles, dim=1)
    return torch.cos(ang).float(), torch.sin(ang).float()


def _apply_rope(x, cos, sin):
    """x [n, H, D]; rotate channel pairs by the per-token angles."""
    xf = x.float().unflatten(-1, (-1, 2))
    a, b = xf[..., 0], xf[..., 1]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(x.dtype)


def _rms(x, w, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def _ln(x):
    return F.layer_norm(x.float(), (x.shape[-1],), eps=1e-6).to(x.dtype)


def _modulate(x, shift, scale):
    return x * (1 + scale) + shift


def _timestep_embedding(t: torch.Tensor, dim: int = 256) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat((torch.cos(args), torch.sin(args)), dim=-1)


class _Weights:
    """Random weights: N(0, 1/fan_in) matrices, zero biases, unit norm weights."""

    def __init__(self, device, dtype, generator):
        self.device, self.dtype, self.g = device, dtype, generator

    def linear(self, out_f, in_f):
        w = torch.randn(out_f, in_f, device=self.device, dtype=torch.float32, generator=self.g)
        return (w / math.sqrt(in_f)).to(self.dtype), torch.zeros(out_f, device=self.device, dtype=self.dtype)

    def ones(self, n):
        return torch.ones(n, device=self.device, dtype=self.dtype)


class HunyuanDiT:
    """``forward(latent, text, t, pooled, guidance) -> velocity tokens``.

    ``latent`` [C_in, T, Hl, Wl] (the full latent on every rank), ``text`` [Nt, text_dim],
    ``pooled`` [vec_dim]; ``attention(block_index, q_img, k_img, v_img, q_txt, k_txt, v_txt)``
    returns ``(o_img, o_txt)`` with ``q_img`` [n_local, H, D] and ``q_txt`` [Nt, H, D].
    Returns this rank's video tokens of the predicted velocity, [n_local, patch_volume * C_in]."""

    def __init__(self, config: HunyuanDiTConfig, device, dtype=torch.bfloat16, seed: int = 0):
        config.validate()
        self.cfg = config
        self.device, self.dtype = device, dtype
        g = torch.Generator(device=device).manual_seed(seed)
        W = _Weights(device, dtype, g)
        c, mlp = config.hidden, int(config.hidden * config.mlp_ratio)
        pv = config.patch[0] * config.patch[1] * config.patch[2]
        self.patch_in = W.linear(c, config.in_channels * pv)
        self.txt_in = W.linear(c, config.text_dim)
        self.time_in = (W.linear(c, 256), W.linear(c, c))
        self.guid_in = (W.linear(c, 256), W.linear(c, c))
        self.vec_in = (W.linear(c, config.vec_dim), W.linear(c, c))
        self.double = []
        for _ in range(config.double_blocks):
            blk = {}
            for s in ("img", "txt"):
                blk[s] = dict(mod=W.linear(6 * c, c), qkv=W.linear(3 * c, c), proj=W.linear(c, c),
                              qn=W.ones(config.head_dim), kn=W.ones(config.head_dim),
                              fc1=W.linear(mlp, c), fc2=W.linear(c, mlp))
            self.double.append(blk)
        self.single = [dict(mod=W.linear(3 * c, c), lin1=W.linear(3 * c + mlp, c), lin2=W.linear(c, c + mlp),
                            qn=W.ones(config.head_dim), kn=W.ones(config.head_dim))
                       for _ in range(config.single_blocks)]
        self.final_mod = W.linear(2 * c, c)
        self.final = W.linear(config.in_channels * pv, c)

    # -- pieces ------------------------------------------------------------------
    @staticmethod
    def _lin(x, wb):
        return F.linear(x, wb[0], wb[1])

    def _mlp2(self, x, pair, act=F.silu):
        return self._lin(act(self._lin(x, pair[0])), pair[1])

    def patchify(self, latent):
        """[C, T, Hl, Wl] -> tokens [T * Hl/2 * Wl/2, C * 4] (row-major t, h, w) and the token grid."""
        pt, ph, pw = self.cfg.patch
        c, t, h, w = latent.shape
        x = latent.reshape(c, t // pt, pt, h // ph, ph, w // pw, pw).permute(1, 3, 5, 0, 2, 4, 6)
        return x.reshape((t // pt) * (h // ph) * (w // pw), c * pt * ph * pw), (t // pt, h // ph, w // pw)

    # -- forward -------------------------------------------------------------------
    def forward(self, latent, text, t, pooled, guidance, attention, rank: int = 0, world: int = 1):
        cfg = self.cfg
        tokens, grid = self.patchify(latent.to(self.dtype))
        n = tokens.shape[0]
        if n % world:
            raise ValueError(f"{n} video tokens do not shard over {world} ranks")
        ns = n // world
        pos = torch.arange(rank * ns, (rank + 1) * ns, device=self.device)
        cos, sin = rope_3d(grid, pos, cfg.rope_axes, cfg.rope_theta, self.device)
        img = self._lin(tokens[rank * ns:(rank + 1) * ns], self.patch_in)
        txt = self._lin(text.to(self.dtype), self.txt_in)
        vec = (self._mlp2(_timestep_embedding(t.view(1)).to(self.dtype), self.time_in)
               + self._mlp2(_timestep_embedding(guidance.view(1)).to(self.dtype), self.guid_in)
               + self._mlp2(pooled.to(self.dtype).view(1, -1), self.vec_in)).view(-1)
        svec = F.silu(vec)
        nt = txt.shape[0]
        for i, blk in enumerate(self.double):
            mods = {s: self._lin(svec, blk[s]["mod"]).chunk(6) for s in ("img", "txt")}
            qkv = {}
            for s, x in (("img", img), ("txt", txt)):
                sh1, sc1 = mods[s][0], mods[s][1]
                h = self._lin(_modulate(_ln(x), sh1, sc1), blk[s]["qkv"])
                q, k, v = h.view(x.shape[0], 3, cfg.heads, cfg.head_dim).unbind(1)
                q, k = _rms(q, blk[s]["qn"]), _rms(k, blk[s]["kn"])
                if s == "img":
                    q, k = _apply_rope(q, cos, sin), _apply_rope(k, cos, sin)
                qkv[s] = (q, k, v)
            o_img, o_txt = attention(i, *qkv["img"], *qkv["txt"])
            outs = {"img": o_img, "txt": o_txt}
            new = {}
            for s, x in (("img", img), ("txt", txt)):
                sh1, sc1, g1, sh2, sc2, g2 = mods[s]
                x = x + g1 * self._lin(outs[s].reshape(x.shape[0], cfg.hidden), blk[s]["proj"])
                h = self._lin(_modulate(_ln(x), sh2, sc2), blk[s]["fc1"])
                new[s] = x + g2 * self._lin(F.gelu(h, approximate="tanh"), blk[s]["fc2"])
            img, txt = new["img"], new["txt"]
        mlp = int(cfg.hidden * cfg.mlp_ratio)
        for j, blk in enumerate(self.single):
            sh, sc, g = self._lin(svec, blk["mod"]).chunk(3)
            x = torch.cat((img, txt), dim=0)
            h = self._lin(_modulate(_ln(x), sh, sc), blk["lin1"])
            qkv, m = h.split((3 * cfg.hidden, mlp), dim=-1)
            q, k, v = qkv.view(x.shape[0], 3, cfg.heads, cfg.head_dim).unbind(1)
            q, k = _rms(q, blk["qn"]), _rms(k, blk["kn"])
            q = torch.cat((_apply_rope(q[:ns], cos, sin), q[ns:]))
            k = torch.cat((_apply_rope(k[:ns], cos, sin), k[ns:]))
            o_img, o_txt = attention(len(self.double) + j, q[:ns], k[:ns], v[:ns], q[ns:], k[ns:], v[ns:])
            o = torch.cat((o_img, o_txt), dim=0).reshape(x.shape[0], cfg.hidden)
            x = x + g * self._lin(torch.cat((o, F.gelu(m, approximate="tanh")), dim=-1), blk["lin2"])
            img, txt = x[:ns], x[ns:]
        sh, sc = self._lin(svec, self.final_mod).chunk(2)
        return self._lin(_modulate(_ln(img), sh, sc), self.final)


class JointAttention:
    """The ``attention`` callable of :class:`HunyuanDiT`.

    ``inner(i, q, k, v, video_tokens)`` attends ``[1, h, video + text, D]`` tensors
    (video tokens first) for block ``i``.  With ``group`` of W > 1 ranks the video
    Q/K/V shards are exchanged into head shards first (all video tokens, H/W heads),
    the text rows are sliced to the same heads, and afterwards the video output
    returns to sequence shards while the text rows' heads are all-gathered.
    ``events`` (optional list) collects (start, end) CUDA events around ``inner``."""

    def __init__(self, inner, group=None, events=None):
        self.inner, self.group, self.events = inner, group, events

    def __call__(self, i, q_img, k_img, v_img, q_txt, k_txt, v_txt):
        import torch.distributed as dist

        from .ulysses import head_to_seq, seq_to_head

        world = dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1
        heads = q_txt.shape[1]
        if world > 1:
            rank = dist.get_rank(self.group)
            hs = heads // world
            vid = [seq_to_head(x.unsqueeze(0), self.group) for x in (q_img, k_img, v_img)]
            txt = [x[:, rank * hs:(rank + 1) * hs].transpose(0, 1).unsqueeze(0) for x in (q_txt, k_txt, v_txt)]
        else:
            vid = [x.transpose(0, 1).unsqueeze(0) for x in (q_img, k_img, v_img)]
            txt = [x.transpose(0, 1).unsqueeze(0) for x in (q_txt, k_txt, v_txt)]
        n = vid[0].shape[2]
        q, k, v = (torch.cat((a, b), dim=2).contiguous() for a, b in zip(vid, txt))
        if self.events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        out = self.inner(i, q, k, v, n)
        if self.events is not None:
            ev[1].record()
            self.events.append(ev)
        o_vid, o_txt = out[:, :, :n], out[:, :, n:].contiguous()
        if world > 1:
            o_img = head_to_seq(o_vid.contiguous(), self.group)[0]
            parts = [torch.empty_like(o_txt) for _ in range(world)]
            dist.all_gather(parts, o_txt, group=self.group)
            o_t = torch.cat(parts, dim=1)[0].transpose(0, 1)
        else:
            o_img = o_vid[0].transpose(0, 1)
            o_t = o_txt[0].transpose(0, 1)
        return o_img.contiguous(), o_t.contiguous()


class SparsePRBlocks:
    """``inner`` for :class:`JointAttention`: SparsePR's Hunyuan boundary with one
    ``N8V6Core`` per block (each block keeps its own cross-step state);
    ``prompt_length`` of the text tokens are real, the rest padding."""

    def __init__(self, config, blocks: int, prompt_length: int):
        from .n8_v6 import N8V6Core

        self.config = config
        self.cores = [N8V6Core(config) for _ in range(blocks)]
        self.prompt_length = int(prompt_length)

    def reset(self) -> None:
        """Fresh cores (cold routing on the next call of every block)."""
        from .n8_v6 import N8V6Core

        self.cores = [N8V6Core(self.config) for _ in self.cores]

    def __call__(self, i, q, k, v, video_tokens):
        from .attention import hunyuan_sparse_attention

        return hunyuan_sparse_attention(q, k, v, self.cores[i], video_tokens=video_tokens,
                                        prompt_length=self.prompt_length)
