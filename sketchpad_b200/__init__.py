"""sketchpad_b200 -- B200-native (sm_100a) diffusion-denoiser kernels behind the C ABI of
include/sketchpad_b200.h, with a host API that mirrors rhi-zone/sketchpad's GPU operator
surface (crates/sketchpad-cubecl) and the sketchpad-core signatures it must match.

The kernels live in libsketchpad_b200.so (built from csrc/ by build.py); there is no CPU or
library fallback.  torch supplies device memory, streams and torch.distributed only.
"""
from ._lib import SketchpadError, load as load_library  # noqa: F401
from .attention import (AttentionSetupError, FlashAttentionOptions, attention_flops,  # noqa: F401
                        causal_mask, flash_attention, flash_attention_masked, qkv_attention)
from .groupnorm_silu import (GroupNormSiLuLayer, GroupNormSiLuOptions, groupnorm,  # noqa: F401
                             groupnorm_bytes, groupnorm_silu)
from .layernorm import LayerNorm, layer_norm, layer_norm_modulate  # noqa: F401
from .quantization import (Fp8Config, Fp8Format, Fp8Linear, Fp8Tensor, quantize_fp8)  # noqa: F401
from .quantized_matmul import (GpuQuantizedLinear, GpuQuantType, dequantize_q8_0,  # noqa: F401
                               repack_q8_0, repack_q8_0_host)

__version__ = "0.1.0"
