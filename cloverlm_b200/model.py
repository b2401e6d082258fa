"""CloverLM transformer with every block linear a Quartet-II NVFP4 layer.

The model the reference trains with ``--quartet true`` (src/models/transformer.py:291-620,
src/models/mlp.py:77-120), in the configuration of its 4B run (README.md:30: 29 blocks,
28 heads of 128, ratio 4 -> 7 key/value heads: vocab 32768,
context 2048):

  X = emb(ids)                                   fp32 residual stream
  per block:
    Q, K, V = lq(X), lk(X), lv(X)                Quartet_II_linear, one shared quantization of X
    Q = scale_h * sphere(rope(Q)), K = sphere(rope(K))      (qk_norm; learned per-head scale)
    Y = lo(causal_attention(Q, K, V))            softmax scale 1 (the scale is in Q)
    X = X + rmsnorm_att(Y)                       (out_att_norm; no pre-norms)
    Z = l2(relu(l1(X))^2)                        MLP2L with ReLU^2
    X = X + rmsnorm_mlp(Z)                       (out_mlp_norm)
  logits = rmsnorm_out(X) @ emb.weight^T         (tied embeddings)

Defaults of the reference kept: RoPE with base 1024 on interleaved pairs, sphere norm with
eps 1e-12, RMSNorm eps = fp32 machine epsilon, biases off, dropout 0, weights
N(0, 0.02), norm weights 1, attention scale sqrt(d_head).

B200 layout of the work: the three projections of a block quantize X once
(fusion.shared_input_forward); RoPE + sphere norm + scale is one libq2b kernel per
direction (q2b_rope_norm_fwd / _bwd); each residual RMSNorm writes the fp32 residual,
its bf16 copy and that copy's abs-max in one pass (q2b_add_rmsnorm_amax), so the next
Quartet layer skips its abs-max read; the MLP's ReLU^2 and its abs-max come out of the first
linear's GEMM epilogue and its gradient out of the second linear's dgrad epilogue
(fusion.mlp_relu2); attention is cuDNN's fused
kernel through torch SDPA (a library call, like the reference's FlashAttention);
the tied head and cross-entropy run in row chunks so no full [tokens, vocab]
logit matrix is ever stored.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import _lib
from .fusion import mlp_relu2, shared_input_forward
from .linear import Quartet_II_linear
from .quant import abs_max


@dataclass
class CloverLMConfig:
    vocab_size: int = 32768
    num_blocks: int = 29
    heads: int = 28
    d_head: int = 128
    ratio: int = 4            # query heads per key/value head
    exp_factor: int = 4       # MLP hidden = exp_factor * d
    context: int = 2048
    rope_base: float = 1024.0
    std: float = 0.02
    norm_eps: float = float(torch.finfo(torch.float32).eps)
    tied_embeddings: bool = True

    @property
    def d(self) -> int:
        return self.heads * self.d_head

    @property
    def groups(self) -> int:
        return self.heads // self.ratio

    @property
    def d_hidden(self) -> int:
        return self.exp_factor * self.d

    def linear_flops_per_token(self) -> float:
        """6 * (sum of K*N over the Quartet linears): forward + dgrad + wgrad."""
        d, dkv, dh = self.d, self.groups * self.d_head, self.d_hidden
        return 6.0 * self.num_blocks * (2 * d * d + 2 * d * dkv + 2 * d * dh)

    def train_flops_per_token(self) -> float:
        """Linears + causal attention (fwd 2 GEMMs over half the context, bwd 2.5x) + tied head."""
        attn = 3.5 * 2 * 2 * self.num_blocks * self.d * self.context / 2
        head = 6.0 * self.d * self.vocab_size
        return self.linear_flops_per_token() + attn + head


def rope_table(context: int, d_head: int, base: float, device) -> torch.Tensor:
    """(cos, sin) fp32 [context, d_head/2, 2] as the reference builds them (transformer.py:39-62)."""
    ms = torch.arange(0.0, context, device=device, dtype=torch.float32)
    js = torch.arange(0.0, d_head // 2, device=device, dtype=torch.float32)
    thetas = 1 / base ** (2 * js / d_head)
    phis = ms[:, None] * thetas[None, :]
    return torch.stack((torch.cos(phis), torch.sin(phis)), dim=-1).contiguous()


def _stream(t):
    return _lib.stream_of(t)


# ------------------------------------------------------------------ RoPE + sphere norm

class _RopeNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, table, scale, heads, seq):
        x = x.contiguous()
        rows = x.numel() // (heads * 128)
        out = torch.empty(*x.shape[:-1], heads, 128, dtype=torch.bfloat16, device=x.device)
        norm = torch.empty(rows, heads, dtype=torch.float32, device=x.device)
        sc = None if scale is None else scale.detach().reshape(-1).float().contiguous()
        with torch.cuda.device(x.device):
            _lib.call("q2b_rope_norm_fwd", _lib.ptr(out), _lib.ptr(norm), _lib.ptr(x), _lib.ptr(table),
                      _lib.ptr(sc), rows, heads, seq, _stream(x))
        ctx.save_for_backward(out, norm, table, sc)
        ctx.has_scale = scale is not None
        ctx.scale_shape = None if scale is None else scale.shape
        ctx.heads, ctx.seq, ctx.x_shape = heads, seq, x.shape
        return out

    @staticmethod
    def backward(ctx, gout):
        out, norm, table, sc = ctx.saved_tensors
        gout = gout.to(torch.bfloat16).contiguous()
        rows = out.numel() // (ctx.heads * 128)
        dx = torch.empty(ctx.x_shape, dtype=torch.bfloat16, device=out.device)
        dscale = torch.zeros(ctx.heads, dtype=torch.float32, device=out.device) if ctx.has_scale else None
        with torch.cuda.device(out.device):
            _lib.call("q2b_rope_norm_bwd", _lib.ptr(dx), _lib.ptr(dscale), _lib.ptr(gout), _lib.ptr(out),
                      _lib.ptr(norm), _lib.ptr(table), _lib.ptr(sc), rows, ctx.heads, ctx.seq, _stream(out))
        ds = None if dscale is None else dscale.reshape(ctx.scale_shape)
        return dx, None, ds, None, None


def rope_sphere_norm(x, table, scale, heads: int, seq: int):
    """bf16 [..., heads*128] -> bf16 [..., heads, 128]: scale * normalize(rope(x)) per head."""
    return _RopeNorm.apply(x, table, scale, heads, seq)


# -------------------------------------------------------- residual RMSNorm + abs-max

class _AddRMSNormAmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, w, eps):
        x = x.contiguous()
        y = y.to(torch.bfloat16).contiguous()
        d = x.shape[-1]
        rows = x.numel() // d
        x_out = torch.empty_like(x, dtype=torch.float32)
        xb = torch.empty_like(x, dtype=torch.bfloat16)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        amax = torch.empty((), dtype=torch.float32, device=x.device)
        wc = w.detach().float().contiguous()
        with torch.cuda.device(x.device):
            _lib.call("q2b_add_rmsnorm_amax", _lib.ptr(x_out), _lib.ptr(xb), _lib.ptr(rstd), _lib.ptr(amax),
                      _lib.ptr(x), _lib.ptr(y), _lib.ptr(wc), rows, d, float(eps), _stream(x))
        ctx.save_for_backward(y, rstd, wc)
        ctx.mark_non_differentiable(amax)
        return x_out, xb, amax

    @staticmethod
    def backward(ctx, g32, gb, gamax):
        y, rstd, w = ctx.saved_tensors
        d = y.shape[-1]
        rows = y.numel() // d
        if g32 is None:
            g32 = torch.zeros(y.shape, dtype=torch.float32, device=y.device)
        g32 = g32.float().contiguous()
        gb = None if gb is None else gb.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(g32)
        dy = torch.empty_like(y)
        props = torch.cuda.get_device_properties(y.device)
        parts = max(1, min(rows, 8 * props.multi_processor_count))  # eight blocks per SM keep enough loads in flight
        dw_part = torch.empty(parts, d, dtype=torch.float32, device=y.device)
        with torch.cuda.device(y.device):
            _lib.call("q2b_rmsnorm_bwd", _lib.ptr(dx), _lib.ptr(dy), _lib.ptr(dw_part), parts, _lib.ptr(g32),
                      _lib.ptr(gb), _lib.ptr(y), _lib.ptr(rstd), _lib.ptr(w), rows, d, _stream(y))
        return dx, dy, dw_part.sum(0), None


def add_rmsnorm_amax(x, y, w, eps):
    """(x + rmsnorm(y) * w in fp32, its bf16 copy, abs-max of that copy)."""
    return _AddRMSNormAmax.apply(x, y, w, eps)


# ------------------------------------------------------------ tied head + loss

class _TiedHeadCrossEntropy(torch.autograd.Function):
    """mean cross-entropy of (h @ W^T) against targets, computed in row chunks: each chunk's
    bf16 logits, fp32 log-softmax, gradient and its two GEMMs are done before the next, and
    the gradients w.r.t. h and W are kept for backward (scaled there by the incoming
    gradient), so at most one chunk of logits exists at a time."""

    CHUNK = 4096

    @staticmethod
    def forward(ctx, h, w, targets):
        n, d = h.shape
        hb = h.to(torch.bfloat16)
        wb = w.to(torch.bfloat16)
        dh = torch.empty_like(hb)
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        total = torch.zeros((), dtype=torch.float32, device=h.device)
        inv_n = 1.0 / n
        for s in range(0, n, _TiedHeadCrossEntropy.CHUNK):
            e = min(n, s + _TiedHeadCrossEntropy.CHUNK)
            # bf16 logits; q2b_softmax_xent_bf16 reads them once in fp32, writes each row's
            # loss and replaces the logits by the gradient of the mean loss (bf16)
            g = hb[s:e] @ wb.T
            row_loss = torch.empty(e - s, dtype=torch.float32, device=h.device)
            t = targets[s:e].to(torch.int64).contiguous()
            _lib.call("q2b_softmax_xent_bf16", _lib.ptr(g), _lib.ptr(row_loss), _lib.ptr(t), inv_n, e - s, g.shape[1],
                      _lib.stream_of(g))
            total += row_loss.sum()
            dh[s:e] = g @ wb
            # bf16 operands, fp32 accumulation into dw in the GEMM itself
            dw = torch.addmm(dw, g.T, hb[s:e], out_dtype=torch.float32)
        ctx.save_for_backward(dh, dw)
        ctx.h_dtype = h.dtype
        return total * inv_n

    @staticmethod
    def backward(ctx, gl):
        dh, dw = ctx.saved_tensors
        return (dh.to(ctx.h_dtype) * gl).to(ctx.h_dtype), dw * gl, None


# ------------------------------------------------------------------------- model

class Block(torch.nn.Module):
    def __init__(self, cfg: CloverLMConfig, device=None):
        super().__init__()
        d, dkv = cfg.d, cfg.groups * cfg.d_head
        self.cfg = cfg
        self.lq = Quartet_II_linear(d, d, bias=False, device=device)
        self.lk = Quartet_II_linear(d, dkv, bias=False, device=device)
        self.lv = Quartet_II_linear(d, dkv, bias=False, device=device)
        self.lo = Quartet_II_linear(d, d, bias=False, device=device)
        self.scale = torch.nn.Parameter(torch.full((1, cfg.heads, 1, 1), math.sqrt(cfg.d_head), device=device))
        self.att_norm = torch.nn.Parameter(torch.ones(d, device=device))
        self.l1 = Quartet_II_linear(d, cfg.d_hidden, bias=False, device=device)
        self.l2 = Quartet_II_linear(cfg.d_hidden, d, bias=False, device=device)
        self.mlp_norm = torch.nn.Parameter(torch.ones(d, device=device))

    def forward(self, x, xb, xamax, table):
        cfg = self.cfg
        B, T, _ = x.shape
        q, k, v = shared_input_forward(xb, [self.lq, self.lk, self.lv], input_abs_max=xamax)
        q = rope_sphere_norm(q, table, self.scale, cfg.heads, T)
        k = rope_sphere_norm(k, table, None, cfg.groups, T)
        v = v.view(B, T, cfg.groups, cfg.d_head)
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION],
                         set_priority=True):
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, scale=1.0, enable_gqa=True)
        o = o.transpose(1, 2).reshape(B, T, cfg.d)
        y = self.lo(o)
        x, xb, amax = add_rmsnorm_amax(x, y, self.att_norm, cfg.norm_eps)
        z = mlp_relu2(xb, self.l1, self.l2, input_abs_max=amax)
        return add_rmsnorm_amax(x, z, self.mlp_norm, cfg.norm_eps)


class CloverLM(torch.nn.Module):
    def __init__(self, cfg: CloverLMConfig = CloverLMConfig(), device=None):
        super().__init__()
        self.cfg = cfg
        self.emb = torch.nn.Embedding(cfg.vocab_size, cfg.d, device=device)
        self.blocks = torch.nn.ModuleList([Block(cfg, device) for _ in range(cfg.num_blocks)])
        self.out_norm = torch.nn.Parameter(torch.ones(cfg.d, device=device))
        if not cfg.tied_embeddings:
            self.head = torch.nn.Parameter(torch.empty(cfg.vocab_size, cfg.d, device=device))
        self.reset_parameters()
        self._table = None

    @torch.no_grad()
    def reset_parameters(self, generator: torch.Generator | None = None):
        """N(0, std) for linear and embedding weights (transformer.py:518-541)."""
        for m in self.modules():
            if isinstance(m, (torch.nn.Linear, torch.nn.Embedding)):
                m.weight.normal_(0.0, self.cfg.std, generator=generator)
                if isinstance(m, Quartet_II_linear):
                    m.weight_abs_max = None
        if not self.cfg.tied_embeddings:
            self.head.normal_(0.0, self.cfg.std, generator=generator)

    def head_weight(self):
        return self.emb.weight if self.cfg.tied_embeddings else self.head

    def rope(self, T: int, device) -> torch.Tensor:
        if self._table is None or self._table.shape[0] < T or self._table.device != device:
            self._table = rope_table(max(T, self.cfg.context), self.cfg.d_head, self.cfg.rope_base, device)
        return self._table

    def forward(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Mean next-token cross-entropy of ids [B, T] against targets [B, T] (train loss)."""
        B, T = ids.shape
        table = self.rope(T, ids.device)
        x = F.embedding(ids, self.emb.weight)  # fp32
        xb = x.to(torch.bfloat16)
        amax = abs_max(xb.detach().reshape(-1, self.cfg.d))
        for blk in self.blocks:
            x, xb, amax = blk(x, xb, amax, table)
        with torch.autocast("cuda", enabled=False):
            h = F.rms_norm(x, (self.cfg.d,), self.out_norm, self.cfg.norm_eps)
            return _TiedHeadCrossEntropy.apply(h.reshape(B * T, -1), self.head_weight(), targets.reshape(-1))
