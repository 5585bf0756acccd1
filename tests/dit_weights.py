"""Oracle-side weights of the DiT block harnesses, shared by the CPU wiring test and the GPU
parity test: every quantized Linear of a block decoded to f32 by the oracle."""
import numpy as np

import sketchpad_b200.flux as FX
import sketchpad_b200.wan as WN
from helpers import fp8_linear_f32, q8_linear_f32, split_interleaved

# Reduced widths with the real head_dim 128.  Q8_0 block scales ~ U(1e-4, 4e-4) give weights
# of std ~0.02 (like the Wan FP8 weights), so attention logits stay O(1).  With the config-4
# range (0.001 .. 0.02) the logits reach O(20) at K=256: the softmax is then so peaked that
# rounding q and k to bf16 alone moves outputs by several percent (a property of bf16
# inputs, not of any kernel), and the 2e-2 bar would test the data, not the implementation.
SMALL_FLUX = FX.FluxConfig(hidden_size=256, num_heads=2, max_seq_len=512,
                           weight_scale=(0.0001, 0.0004))


def flux_block_weights(blk, single: bool):
    W = {"modulation": q8_linear_f32(blk.modulation)}
    streams = [("attn.", blk.attn, "ffn.", blk.ffn)] if single else [
        ("img_attn.", blk.img_attn, "img_ffn.", blk.img_ffn),
        ("txt_attn.", blk.txt_attn, "txt_ffn.", blk.txt_ffn)]
    for ap, attn, fp, ffn in streams:
        W[ap + "qkv"], W[ap + "proj"] = q8_linear_f32(attn.qkv), q8_linear_f32(attn.proj)
        W[fp + "gate"], W[fp + "up"] = split_interleaved(q8_linear_f32(ffn.gate_up))
        W[fp + "down"] = q8_linear_f32(ffn.down)
    return W


def wan_block_weights(blk):
    W = {"modulation": fp8_linear_f32(blk.modulation),
         "spatial.to_qkv": fp8_linear_f32(blk.s_qkv), "spatial.to_out": fp8_linear_f32(blk.s_out),
         "temporal.to_qkv": fp8_linear_f32(blk.t_qkv), "temporal.to_out": fp8_linear_f32(blk.t_out),
         "cross.to_q": fp8_linear_f32(blk.c_q), "cross.to_kv": fp8_linear_f32(blk.c_kv),
         "cross.to_out": fp8_linear_f32(blk.c_out), "expert0.down": fp8_linear_f32(blk.down)}
    W["expert0.gate"], W["expert0.up"] = split_interleaved(fp8_linear_f32(blk.gate_up))
    # one expert: the router's softmax is exactly 1 whatever its weights are
    h = blk.cfg.hidden_size
    W["router"] = (np.random.default_rng(5).standard_normal((1, h)).astype(np.float32) * 0.02,
                   np.zeros(1, np.float32))
    return W


SMALL_WAN = WN.WanConfig(hidden_size=256, num_heads=2, intermediate=512, max_spatial_len=64,
                         max_temporal_len=8)


def flux_model_weights(net):
    """(model-level weights, block_weights(kind, i)) of a FluxB200 for oracle.dit.flux_forward;
    block weights are decoded when the oracle asks for them."""
    W = {"img_embed": q8_linear_f32(net.img_embed), "txt_embed": q8_linear_f32(net.txt_embed),
         "time.linear1": q8_linear_f32(net.t1), "time.linear2": q8_linear_f32(net.t2),
         "guidance.linear1": q8_linear_f32(net.g1), "guidance.linear2": q8_linear_f32(net.g2),
         "final.modulation": q8_linear_f32(net.final_mod),
         "final.proj": q8_linear_f32(net.final_proj)}

    def block(kind, i):
        return flux_block_weights(net.double[i], False) if kind == "double" else \
            flux_block_weights(net.single[i], True)
    return W, block


def wan_model_weights(net):
    """(model-level weights, block_weights(i)) of a WanB200 for oracle.dit.wan_forward."""
    W = {"video_embed": fp8_linear_f32(net.video_embed),
         "text_embed": fp8_linear_f32(net.text_embed),
         "time.linear1": fp8_linear_f32(net.t1), "time.linear2": fp8_linear_f32(net.t2),
         "final.modulation": fp8_linear_f32(net.final_mod),
         "final.proj": fp8_linear_f32(net.final_proj)}
    return W, lambda i: wan_block_weights(net.blocks[i])
