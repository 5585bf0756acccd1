"""CPU restatement of the reference's Flux and Wan transformer blocks (fp32).

TEST INFRASTRUCTURE ONLY (the checker for the GPU DiT block harnesses).  Built on the C++
oracle kernels (linear, attention, layernorm, activation) plus numpy reshapes.  Follows
rhi-zone/sketchpad:
  crates/sketchpad-core/src/rope.rs:60-94      RotaryEmbedding::with_base (cos/sin tables,
                                               each frequency repeated for its pair)
  crates/sketchpad-core/src/rope.rs:116-170    forward / apply_rotary / rotate_half
  crates/sketchpad-core/src/glu.rs:91-96       SwiGluFfn::forward
  crates/sketchpad-core/src/layernorm.rs:63-73 LayerNorm (unbiased variance, gamma 1, beta 0)
  crates/sketchpad-dit/src/flux.rs:325-422     FluxAttention::forward
  crates/sketchpad-dit/src/flux.rs:450-517     FluxDoubleBlock::forward
  crates/sketchpad-dit/src/flux.rs:573-607     FluxSingleBlock::forward
  crates/sketchpad-dit/src/wan.rs:330-337      WanExpert::forward
  crates/sketchpad-dit/src/wan.rs:351-402      WanAttention::forward
  crates/sketchpad-dit/src/wan.rs:418-461      WanCrossAttention::forward
  crates/sketchpad-dit/src/wan.rs:489-573      WanBlock::forward
  crates/sketchpad-dit/src/wan.rs:576-601      WanBlock::forward_moe (dense softmax routing)
Weights are passed in as f32 arrays ``{name: (w [N, K], b [N] or None)}`` (Linear stores
[K, N] in burn; y = x W^T + b is the same product).
"""
from __future__ import annotations

import math

import numpy as np

from . import activation, attention, layernorm, linear_nt


def rope_tables(head_dim: int, max_seq_len: int, base: float = 10000.0):
    """rope.rs:60-94: inv_freq[i] = 1 / base^(2i/d); angles = pos * inv_freq; each value
    repeated for its (even, odd) pair -> cos, sin [max_seq_len, head_dim]."""
    half = head_dim // 2
    inv = np.array([1.0 / np.float32(base) ** np.float32((2 * i) / head_dim) for i in range(half)],
                   np.float32)
    ang = np.arange(max_seq_len, dtype=np.float32)[:, None] * inv[None, :]
    return (np.repeat(np.cos(ang), 2, axis=1).astype(np.float32),
            np.repeat(np.sin(ang), 2, axis=1).astype(np.float32))


def rope_apply(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, start: int = 0) -> np.ndarray:
    """rope.rs:145-170 on x [B, H, S, D]: x*cos + rotate_half(x)*sin with
    rotate_half([x0, x1, x2, x3, ...]) = [-x1, x0, -x3, x2, ...]."""
    S, D = x.shape[-2:]
    pairs = x.reshape(x.shape[:-1] + (D // 2, 2))
    rot = np.stack((-pairs[..., 1], pairs[..., 0]), axis=-1).reshape(x.shape)
    return (x * cos[start:start + S] + rot * sin[start:start + S]).astype(np.float32)


def _lin(x, wb):
    w, b = wb
    return linear_nt(x, w, b)


def _ln(x):
    n = x.shape[-1]
    return layernorm(x, np.ones(n, np.float32), np.zeros(n, np.float32), 1e-5)


def _silu(x):
    return activation(x, "silu")


def _sdpa(q, k, v, head_dim):
    """softmax(Q K^T * d^-1/2) V over [B, H, S, D] (flux.rs:412-415, wan.rs:391-394)."""
    return attention(q, k, v, scale=1.0 / math.sqrt(head_dim))


def swiglu(x, W, prefix):
    """glu.rs:91-96: down(silu(gate(x)) * up(x))."""
    return _lin(_silu(_lin(x, W[prefix + "gate"])) * _lin(x, W[prefix + "up"]), W[prefix + "down"])


def _heads(t, b, s, H, D):
    return t.reshape(b, s, H, D).transpose(0, 2, 1, 3)


def flux_attention(x, W, prefix, H, D, cos, sin, cross=None):
    """flux.rs:325-422.  RoPE (offset 0) on this stream's q and k only; with `cross`, K/V are
    cat(self, cross through the SAME qkv Linear, no RoPE) along the sequence."""
    b, s, _ = x.shape
    qkv = _lin(x, W[prefix + "qkv"]).reshape(b, s, 3, H, D)
    q = qkv[:, :, 0].transpose(0, 2, 1, 3)
    k = qkv[:, :, 1].transpose(0, 2, 1, 3)
    v = qkv[:, :, 2].transpose(0, 2, 1, 3)
    q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
    if cross is not None:
        c = cross.shape[1]
        cq = _lin(cross, W[prefix + "qkv"]).reshape(b, c, 3, H, D)
        k = np.concatenate([k, cq[:, :, 1].transpose(0, 2, 1, 3)], axis=2)
        v = np.concatenate([v, cq[:, :, 2].transpose(0, 2, 1, 3)], axis=2)
    o = _sdpa(q, k, v, D).transpose(0, 2, 1, 3).reshape(b, s, H * D)
    return _lin(o, W[prefix + "proj"])


def flux_double_block(img, txt, cond, W, H, D, cos, sin):
    """flux.rs:450-517.  mod = modulation(cond) -> [b, 1, 6, hidden]: (shift, scale, gate) for
    the image stream, then for the text stream.  The text stream attends to the image stream
    AFTER its update, and each stream's gate scales both of its residual branches."""
    b, _, h = img.shape
    m = _lin(cond, W["modulation"]).reshape(b, 1, 6, h)
    shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
    xn = (1.0 + scale) * _ln(img) + shift
    img = img + gate * flux_attention(xn, W, "img_attn.", H, D, cos, sin, cross=txt)
    img = img + gate * swiglu(_ln(img), W, "img_ffn.")
    shift, scale, gate = m[:, :, 3], m[:, :, 4], m[:, :, 5]
    xn = (1.0 + scale) * _ln(txt) + shift
    txt = txt + gate * flux_attention(xn, W, "txt_attn.", H, D, cos, sin, cross=img)
    txt = txt + gate * swiglu(_ln(txt), W, "txt_ffn.")
    return img.astype(np.float32), txt.astype(np.float32)


def flux_single_block(x, cond, W, H, D, cos, sin):
    """flux.rs:573-607: one (shift, scale, gate); the FFN branch uses the plain norm."""
    b, _, h = x.shape
    m = _lin(cond, W["modulation"]).reshape(b, 1, 3, h)
    shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
    xn = (1.0 + scale) * _ln(x) + shift
    x = x + gate * flux_attention(xn, W, "attn.", H, D, cos, sin)
    return (x + gate * swiglu(_ln(x), W, "ffn.")).astype(np.float32)


def wan_attention(x, W, prefix, H, D, cos, sin):
    """wan.rs:351-402 over x [batch', seq', hidden]."""
    b, s, _ = x.shape
    qkv = _lin(x, W[prefix + "to_qkv"]).reshape(b, s, 3, H, D)
    q = qkv[:, :, 0].transpose(0, 2, 1, 3)
    k = qkv[:, :, 1].transpose(0, 2, 1, 3)
    v = qkv[:, :, 2].transpose(0, 2, 1, 3)
    q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
    o = _sdpa(q, k, v, D).transpose(0, 2, 1, 3).reshape(b, s, H * D)
    return _lin(o, W[prefix + "to_out"])


def wan_cross_attention(x, context, W, H, D):
    """wan.rs:418-461: q from x, k/v from the text context, no RoPE."""
    b, s, _ = x.shape
    c = context.shape[1]
    q = _heads(_lin(x, W["cross.to_q"]), b, s, H, D)
    kv = _lin(context, W["cross.to_kv"]).reshape(b, c, 2, H, D)
    k = kv[:, :, 0].transpose(0, 2, 1, 3)
    v = kv[:, :, 1].transpose(0, 2, 1, 3)
    o = _sdpa(q, k, v, D).transpose(0, 2, 1, 3).reshape(b, s, H * D)
    return _lin(o, W["cross.to_out"])


def wan_block(x, cond, context, W, nt, nh, nw, H, D, spatial_rope, temporal_rope):
    """wan.rs:489-573.  x [b, nt*nh*nw, hidden] (frame-major).  mod = modulation(cond) ->
    [b, 8, hidden] = (shift_i, scale_i) for the four sub-layers; no residual gates."""
    b, S, h = x.shape
    hw = nh * nw
    m = _lin(cond, W["modulation"]).reshape(b, 8, h)
    sh = lambda i: m[:, i:i + 1]  # noqa: E731  [b, 1, hidden]
    # spatial attention: [b, T*HW, h] -> [b*T, HW, h]
    xn = (1.0 + sh(1)) * _ln(x) + sh(0)
    out = wan_attention(xn.reshape(b * nt, hw, h), W, "spatial.", H, D, *spatial_rope)
    x = x + out.reshape(b, S, h)
    # temporal attention: [b, T, HW, h] -> swap(1,2) -> [b*HW, T, h]
    xn = (1.0 + sh(3)) * _ln(x) + sh(2)
    xt = xn.reshape(b, nt, hw, h).transpose(0, 2, 1, 3).reshape(b * hw, nt, h)
    out = wan_attention(xt, W, "temporal.", H, D, *temporal_rope)
    x = x + out.reshape(b, hw, nt, h).transpose(0, 2, 1, 3).reshape(b, S, h)
    # text cross-attention
    xn = (1.0 + sh(5)) * _ln(x) + sh(4)
    x = x + wan_cross_attention(xn, context, W, H, D)
    # MoE FFN (wan.rs:576-601): softmax router over the experts, dense weighted sum
    xn = (1.0 + sh(7)) * _ln(x) + sh(6)
    logits = _lin(xn, W["router"])
    e = np.exp(logits - logits.max(axis=-1, keepdims=True))
    probs = e / e.sum(axis=-1, keepdims=True)
    moe = np.zeros_like(x)
    n_exp = logits.shape[-1]
    for i in range(n_exp):
        gate = _silu(_lin(xn, W[f"expert{i}.gate"]))
        moe = moe + _lin(gate * _lin(xn, W[f"expert{i}.up"]), W[f"expert{i}.down"]) * probs[..., i:i + 1]
    return (x + moe).astype(np.float32)


__all__ = ["rope_tables", "rope_apply", "swiglu", "flux_attention", "flux_double_block",
           "flux_single_block", "wan_attention", "wan_cross_attention", "wan_block"]
