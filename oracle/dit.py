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
  crates/sketchpad-dit/src/flux.rs:199-247     timestep_freqs / TimestepEmbedding::forward_scalar
  crates/sketchpad-dit/src/flux.rs:620-636     FinalLayer::forward
  crates/sketchpad-dit/src/flux.rs:686-741     Flux::forward
  crates/sketchpad-core/src/dit.rs:299-345     PatchEmbed::forward / unpatchify
  crates/sketchpad-dit/src/wan.rs:188-221      wan_timestep_freqs / WanTimestepEmbed
  crates/sketchpad-dit/src/wan.rs:613-627      WanFinalLayer::forward
  crates/sketchpad-dit/src/wan.rs:661-757      Wan::patchify / unpatchify / forward
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


def flux_attention(x, W, prefix, H, D, cos, sin, cross=None, given=None, rows=None):
    """flux.rs:325-422.  RoPE (offset 0) on this stream's q and k only; with `cross`, K/V are
    cat(self, cross through the SAME qkv Linear, no RoPE) along the sequence.

    given: optional (q [b, s, H*D], k [b, s+c, H*D], v [b, s+c, H*D]) -- the attention inputs
    (after RoPE and concatenation) taken from another implementation.  With them the oracle
    skips its own qkv projection and evaluates the attention and everything after it in f32
    from those values: a parity check of one stage fed the previous stage's rounded output.
    rows: optional query-row indices; only those output rows are computed (K and V still
    cover every token), which keeps full-width checks affordable."""
    b, s, _ = x.shape
    if given is not None:
        gq, gk, gv = (np.asarray(t, np.float32) for t in given)
        if rows is not None:
            gq = gq[:, rows]
        q, k, v = (_heads(t, b, t.shape[1], H, D) for t in (gq, gk, gv))
    else:
        qkv = _lin(x, W[prefix + "qkv"]).reshape(b, s, 3, H, D)
        q = qkv[:, :, 0].transpose(0, 2, 1, 3)
        k = qkv[:, :, 1].transpose(0, 2, 1, 3)
        v = qkv[:, :, 2].transpose(0, 2, 1, 3)
        q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        if rows is not None:
            q = np.ascontiguousarray(q[:, :, rows])
        if cross is not None:
            c = cross.shape[1]
            cq = _lin(cross, W[prefix + "qkv"]).reshape(b, c, 3, H, D)
            k = np.concatenate([k, cq[:, :, 1].transpose(0, 2, 1, 3)], axis=2)
            v = np.concatenate([v, cq[:, :, 2].transpose(0, 2, 1, 3)], axis=2)
    o = _sdpa(np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v), D)
    o = o.transpose(0, 2, 1, 3).reshape(b, q.shape[2], H * D)
    return _lin(o, W[prefix + "proj"])


def flux_double_block(img, txt, cond, W, H, D, cos, sin, given=None, img_rows=None,
                      txt_rows=None):
    """flux.rs:450-517.  mod = modulation(cond) -> [b, 1, 6, hidden]: (shift, scale, gate) for
    the image stream, then for the text stream.  The text stream attends to the image stream
    AFTER its update, and each stream's gate scales both of its residual branches.
    given: optional {"img_attn.": (q, k, v), "txt_attn.": (q, k, v)} (see flux_attention).
    img_rows / txt_rows: compute only those output rows of each stream (the text stream's
    K/V need the whole updated image stream, so img_rows requires given["txt_attn."])."""
    given = given or {}
    if img_rows is not None and "txt_attn." not in given:
        raise ValueError("img_rows needs the text stream's attention inputs in `given`")
    b, _, h = img.shape
    ri = slice(None) if img_rows is None else np.asarray(img_rows)
    rt = slice(None) if txt_rows is None else np.asarray(txt_rows)
    m = _lin(cond, W["modulation"]).reshape(b, 1, 6, h)
    shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
    xn = (1.0 + scale) * _ln(img) + shift
    img = img[:, ri] + gate * flux_attention(xn, W, "img_attn.", H, D, cos, sin, cross=txt,
                                             given=given.get("img_attn."), rows=img_rows)
    img = img + gate * swiglu(_ln(img), W, "img_ffn.")
    shift, scale, gate = m[:, :, 3], m[:, :, 4], m[:, :, 5]
    xn = (1.0 + scale) * _ln(txt) + shift
    txt = txt[:, rt] + gate * flux_attention(xn, W, "txt_attn.", H, D, cos, sin, cross=img,
                                             given=given.get("txt_attn."), rows=txt_rows)
    txt = txt + gate * swiglu(_ln(txt), W, "txt_ffn.")
    return img.astype(np.float32), txt.astype(np.float32)


def flux_single_block(x, cond, W, H, D, cos, sin, given=None, rows=None):
    """flux.rs:573-607: one (shift, scale, gate); the FFN branch uses the plain norm.
    given: optional {"attn.": (q, k, v)} (see flux_attention); rows: output rows to compute."""
    given = given or {}
    b, _, h = x.shape
    r = slice(None) if rows is None else np.asarray(rows)
    m = _lin(cond, W["modulation"]).reshape(b, 1, 3, h)
    shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
    xn = (1.0 + scale) * _ln(x) + shift
    x = x[:, r] + gate * flux_attention(xn, W, "attn.", H, D, cos, sin, given=given.get("attn."),
                                        rows=rows)
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


# ------------------------------------------------------------------------------------------
# whole-model forwards
# ------------------------------------------------------------------------------------------
def timestep_freqs(dim: int, log_base: float) -> np.ndarray:
    """flux.rs:199-207 (log_base = ln 2, as the reference writes it) and wan.rs:188-196
    (log_base = ln 10000): freqs[i] = exp(-log_base / (half - 1) * i), all in f32."""
    half = dim // 2
    emb_scale = np.float32(-log_base) / np.float32(half - 1)
    return np.exp(emb_scale * np.arange(half, dtype=np.float32)).astype(np.float32)


def timestep_embedding(t: float, freqs, l1, l2):
    """forward_scalar (flux.rs:234-247, wan.rs:213-221): angles = freqs * t in f32,
    emb = [sin(angles), cos(angles)] as [1, dim], then linear2(silu(linear1(emb)))."""
    a = (freqs * np.float32(t)).astype(np.float32)
    emb = np.concatenate([np.sin(a), np.cos(a)]).astype(np.float32)[None]
    return _lin(_silu(_lin(emb, l1)), l2)


def flux_patch_embed(latents, ps: int):
    """dit.rs:300-322 without the projection: reshape [B, C, ph, ps, pw, ps], swap_dims(2, 4),
    swap_dims(3, 5), reshape [B, ph*pw, C*ps*ps] -- the element order the two swaps give,
    followed literally."""
    B, C, H, Wd = latents.shape
    ph, pw = H // ps, Wd // ps
    x = latents.reshape(B, C, ph, ps, pw, ps)
    x = np.swapaxes(np.swapaxes(x, 2, 4), 3, 5)
    return np.ascontiguousarray(x).reshape(B, ph * pw, C * ps * ps).astype(np.float32)


def flux_unpatchify(x, ps: int, H: int, Wd: int, C: int):
    """dit.rs:326-345: reshape [B, ph, pw, C, ps, ps], swap_dims(2, 4), swap_dims(3, 5),
    reshape [B, C, H, W] (literal element order)."""
    B = x.shape[0]
    ph, pw = H // ps, Wd // ps
    y = x.reshape(B, ph, pw, C, ps, ps)
    y = np.swapaxes(np.swapaxes(y, 2, 4), 3, 5)
    return np.ascontiguousarray(y).reshape(B, C, H, Wd).astype(np.float32)


def _final_layer(x, cond, W, prefix):
    """flux.rs:620-636 / wan.rs:613-627: (shift, scale) = modulation(cond); proj((1 + scale) *
    LN(x) + shift)."""
    b, _, h = x.shape
    m = _lin(cond, W[prefix + "modulation"]).reshape(b, 1, 2 * h)
    shift, scale = m[..., :h], m[..., h:]
    return _lin((1.0 + scale) * _ln(x) + shift, W[prefix + "proj"])


def flux_forward(latents, timestep, txt_embeds, W, block_weights, num_double, num_single,
                 H, D, patch_size, cos, sin, guidance=None):
    """flux.rs:686-741.  W holds the model-level Linears ("img_embed", "txt_embed",
    "time.linear1/2", optionally "guidance.linear1/2", "final.modulation", "final.proj");
    block_weights(kind, i) returns the weights of double / single block i (decoded on demand,
    so only one block's f32 weights are held at a time)."""
    B, C, Hh, Wd = latents.shape
    img = _lin(flux_patch_embed(latents, patch_size), W["img_embed"])
    n_img = img.shape[1]
    txt = _lin(txt_embeds, W["txt_embed"])
    cond = timestep_embedding(timestep, timestep_freqs(W["time.linear1"][0].shape[1],
                                                       math.log(2.0)),
                              W["time.linear1"], W["time.linear2"])
    if guidance is not None and "guidance.linear1" in W:
        cond = cond + timestep_embedding(
            guidance, timestep_freqs(W["guidance.linear1"][0].shape[1], math.log(2.0)),
            W["guidance.linear1"], W["guidance.linear2"])
    for i in range(num_double):
        img, txt = flux_double_block(img, txt, cond, block_weights("double", i), H, D, cos, sin)
    x = np.concatenate([img, txt], axis=1)
    for i in range(num_single):
        x = flux_single_block(x, cond, block_weights("single", i), H, D, cos, sin)
    out = _final_layer(x[:, :n_img], cond, W, "final.")
    return flux_unpatchify(out, patch_size, Hh, Wd, C)


def wan_patchify(latents, ps: int):
    """wan.rs:661-689 without the projection: [B, C, T, H, W] -> permute [B, T, C, H, W] ->
    [B*T, C, nh, ps, nw, ps] -> permute [B*T, nh, nw, C, ps, ps] -> [B, T*nh*nw, C*ps*ps]."""
    B, C, T, Hh, Wd = latents.shape
    nh, nw = Hh // ps, Wd // ps
    x = latents.transpose(0, 2, 1, 3, 4).reshape(B * T, C, nh, ps, nw, ps)
    x = x.transpose(0, 2, 4, 1, 3, 5)
    return np.ascontiguousarray(x).reshape(B, T * nh * nw, C * ps * ps).astype(np.float32)


def wan_unpatchify(x, nt: int, nh: int, nw: int, C: int, ps: int):
    """wan.rs:691-718: [B, T*nh*nw, C*ps*ps] -> [B*T, nh, nw, C, ps, ps] -> permute
    [B*T, C, nh, ps, nw, ps] -> [B, T, C, H, W] -> permute [B, C, T, H, W]."""
    B = x.shape[0]
    y = x.reshape(B * nt, nh, nw, C, ps, ps).transpose(0, 3, 1, 4, 2, 5)
    y = np.ascontiguousarray(y).reshape(B, nt, C, nh * ps, nw * ps).transpose(0, 2, 1, 3, 4)
    return np.ascontiguousarray(y).astype(np.float32)


def wan_forward(latents, timestep, text_embeds, W, block_weights, num_blocks, H, D,
                patch_size, spatial_rope, temporal_rope):
    """wan.rs:720-757 (temporal patch 1).  W: "video_embed", "text_embed", "time.linear1/2",
    "final.modulation", "final.proj"; block_weights(i) returns block i's weights."""
    B, C, T, Hh, Wd = latents.shape
    nh, nw = Hh // patch_size, Wd // patch_size
    x = _lin(wan_patchify(latents, patch_size), W["video_embed"])
    context = _lin(text_embeds, W["text_embed"])
    cond = timestep_embedding(timestep, timestep_freqs(W["time.linear1"][0].shape[1],
                                                       math.log(10000.0)),
                              W["time.linear1"], W["time.linear2"])
    for i in range(num_blocks):
        x = wan_block(x, cond, context, block_weights(i), T, nh, nw, H, D, spatial_rope,
                      temporal_rope)
    out = _final_layer(x, cond, W, "final.")
    return wan_unpatchify(out, T, nh, nw, C, patch_size)


__all__ = ["rope_tables", "rope_apply", "swiglu", "flux_attention", "flux_double_block",
           "flux_single_block", "wan_attention", "wan_cross_attention", "wan_block",
           "timestep_freqs", "timestep_embedding", "flux_patch_embed", "flux_unpatchify",
           "flux_forward", "wan_patchify", "wan_unpatchify", "wan_forward"]
