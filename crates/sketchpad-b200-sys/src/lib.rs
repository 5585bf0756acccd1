//! Raw FFI to libsketchpad_b200.so: every entry point of include/sketchpad_b200.h, the C ABI
//! of the B200-native (sm_100a) kernels of sketchpad's diffusion-denoiser hot path.
//!
//! Conventions (as in the header): device pointers unless a name ends in `_host`; every
//! launch is asynchronous on `stream` (a `cudaStream_t`, null = the legacy default stream);
//! outputs are allocated by the caller; the return value is a status (`SP_OK` = 0, negative
//! = error) and `sp_last_error()` describes the calling thread's last failure; strides are
//! in elements.  The safe layer keeping the reference's operator signatures is the
//! `sketchpad-b200` crate.
#![allow(non_camel_case_types)]
#![no_std]

use core::ffi::{c_char, c_double, c_float, c_int, c_void};

pub const SP_ABI_VERSION: c_int = 1;

// sp_status
pub const SP_OK: c_int = 0;
pub const SP_ERR_INVALID_ARG: c_int = -1;
pub const SP_ERR_SHAPE: c_int = -2;
pub const SP_ERR_DTYPE: c_int = -3;
pub const SP_ERR_ALIGN: c_int = -4;
pub const SP_ERR_LAUNCH: c_int = -5;
pub const SP_ERR_WORKSPACE: c_int = -6;
pub const SP_ERR_DEVICE: c_int = -7;
pub const SP_ERR_COMM: c_int = -8;

// sp_dtype
pub const SP_F32: c_int = 0;
pub const SP_F16: c_int = 1;
pub const SP_BF16: c_int = 2;

// sp_act
pub const SP_ACT_NONE: c_int = 0;
pub const SP_ACT_SILU: c_int = 1;

// sp_glu_kind
pub const SP_GLU_GEGLU: c_int = 0;
pub const SP_GLU_SWIGLU: c_int = 1;

// sp_kquant_format
pub const SP_QK_Q2_K: c_int = 10;
pub const SP_QK_Q3_K: c_int = 11;
pub const SP_QK_Q4_K: c_int = 12;

// sp_fp8_scale_mode
pub const SP_FP8_PER_TENSOR: c_int = 0;
pub const SP_FP8_PER_CHANNEL: c_int = 1;
pub const SP_FP8_GIVEN_SCALE: c_int = 2;

// sp_container
pub const SP_CONTAINER_GGUF: c_int = 1;
pub const SP_CONTAINER_SAFETENSORS: c_int = 2;

// sp_tensor_type (GGUF block types: SP_T_GGML_BASE + ggml type id)
pub const SP_T_F32: c_int = 0;
pub const SP_T_F16: c_int = 1;
pub const SP_T_BF16: c_int = 2;
pub const SP_T_F8_E4M3: c_int = 3;
pub const SP_T_F8_E5M2: c_int = 4;
pub const SP_T_F64: c_int = 5;
pub const SP_T_I8: c_int = 6;
pub const SP_T_U8: c_int = 7;
pub const SP_T_I16: c_int = 8;
pub const SP_T_I32: c_int = 9;
pub const SP_T_I64: c_int = 10;
pub const SP_T_BOOL: c_int = 11;
pub const SP_T_GGML_BASE: c_int = 100;

extern "C" {
    // -- library, errors, device watchdog
    pub fn sp_abi_version() -> c_int;
    pub fn sp_last_error() -> *const c_char;
    pub fn sp_watchdog_read_and_clear(stream: *mut c_void, code_out: *mut c_int) -> c_int;
    // -- flash attention: sketchpad_cubecl::flash_attention / flash_attention_masked
    //    (crates/sketchpad-cubecl/src/attention.rs:97, :119); a bounded-wait check
    pub fn sp_flash_attn_fwd(
        q: *const c_void, k: *const c_void, v: *const c_void, mask: *const c_float,
        mask_row_stride: i64, out: *mut c_void, b: i64, h: i64, sq: i64, skv: i64, d: i64,
        dv: i64, q_strides: *const i64, k_strides: *const i64, v_strides: *const i64,
        o_strides: *const i64, dtype_in: c_int, dtype_out: c_int, causal: c_int,
        scale: c_float, stream: *mut c_void
    ) -> c_int;
    pub fn sp_flash_attn_fwd_wait_test(
        q: *const c_void, k: *const c_void, v: *const c_void, out: *mut c_void, b: i64, h: i64,
        s: i64, d: i64, skip_kv_tile: c_int, wait_budget_cycles: i64, stream: *mut c_void
    ) -> c_int;
    // -- GroupNorm (+ SiLU): sketchpad_cubecl::groupnorm_silu / groupnorm
    //    (crates/sketchpad-cubecl/src/groupnorm_silu.rs:232, :323)
    pub fn sp_groupnorm_act_workspace_size(
        b: i64, c: i64, h: i64, w: i64, x_strides: *const i64, groups: i64, dtype: c_int
    ) -> usize;
    pub fn sp_groupnorm_act(
        x: *const c_void, gamma: *const c_void, beta: *const c_void, y: *mut c_void, b: i64,
        c: i64, h: i64, w: i64, x_strides: *const i64, groups: i64, eps: c_float, act: c_int,
        dtype: c_int, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void
    ) -> c_int;
    pub fn sp_groupnorm_act_output_strides(
        b: i64, c: i64, h: i64, w: i64, x_strides: *const i64, y_strides: *mut i64
    ) -> c_int;
    pub fn sp_groupnorm_add_act(
        x: *const c_void, x_add: *const c_void, gamma: *const c_void, beta: *const c_void,
        y: *mut c_void, b: i64, c: i64, h: i64, w: i64, x_strides: *const i64, groups: i64,
        eps: c_float, act: c_int, dtype: c_int, workspace: *mut c_void, workspace_bytes: usize,
        stream: *mut c_void
    ) -> c_int;
    pub fn sp_groupnorm_act_noalloc_max_scratch_bytes() -> usize;
    pub fn sp_groupnorm_act_noalloc(
        x: *const c_void, gamma: *const c_void, beta: *const c_void, y: *mut c_void, b: i64,
        c: i64, h: i64, w: i64, x_strides: *const i64, groups: i64, eps: c_float, act: c_int,
        dtype: c_int, stream: *mut c_void
    ) -> c_int;
    // -- fusions around the path (GLU gates, residual adds)
    pub fn sp_glu_gate(
        x: *const c_void, y: *mut c_void, rows: i64, f: i64, x_row_stride: i64,
        y_row_stride: i64, kind: c_int, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_add_bias_residual(
        y: *const c_void, r: *const c_void, bias: *const c_void, out: *mut c_void, rows: i64,
        c: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    // -- Q8_0 / K-quant weights: dequantize_q8_0 and GpuQuantizedLinear
    //    (crates/sketchpad-cubecl/src/quantized_matmul.rs:376, :655-767); bf16 linears
    pub fn sp_q8_0_repack_host(
        gguf_host: *const u8, nbytes: usize, out_f: i64, in_f: i64, q_host: *mut i8,
        scale_host: *mut u16
    ) -> c_int;
    pub fn sp_q8_0_repack(
        gguf: *const c_void, nbytes: usize, out_f: i64, in_f: i64, q: *mut c_void,
        scale: *mut c_void, stream: *mut c_void
    ) -> c_int;
    pub fn sp_q8_0_dequant(
        q: *const c_void, scale: *const c_void, out_f: i64, in_f: i64, out: *mut c_void,
        out_dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_kquant_repack_host(
        fmt: c_int, gguf_host: *const u8, nbytes: usize, out_f: i64, in_f: i64,
        qpack_host: *mut u8, a_host: *mut c_float, b_host: *mut c_float
    ) -> c_int;
    pub fn sp_kquant_dequant(
        fmt: c_int, qpack: *const c_void, a: *const c_float, b: *const c_float, out_f: i64,
        in_f: i64, out: *mut c_void, out_dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_kquant_linear(
        fmt: c_int, x: *const c_void, qpack: *const c_void, a: *const c_float,
        b: *const c_float, bias: *const c_void, y: *mut c_void, m: i64, n: i64, k: i64,
        dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_quant_linear_set_pairing(mode: c_int) -> c_int;
    pub fn sp_q8_0_linear(
        x: *const c_void, q: *const c_void, scale: *const c_void, bias: *const c_void,
        y: *mut c_void, m: i64, n: i64, k: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_q8_0_linear_gated(
        x: *const c_void, q: *const c_void, scale: *const c_void, bias: *const c_void,
        gate: *const c_void, residual: *const c_void, y: *mut c_void, m: i64, n: i64, k: i64,
        dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_bf16_linear(
        x: *const c_void, w: *const c_void, bias: *const c_void, y: *mut c_void, m: i64,
        n: i64, k: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_bf16_linear_gated(
        x: *const c_void, w: *const c_void, bias: *const c_void, gate: *const c_void,
        residual: *const c_void, y: *mut c_void, m: i64, n: i64, k: i64, dtype: c_int,
        stream: *mut c_void
    ) -> c_int;
    pub fn sp_bf16_linear_glu(
        x: *const c_void, w: *const c_void, bias: *const c_void, y: *mut c_void, m: i64,
        n: i64, k: i64, glu_kind: c_int, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    // -- FP8 e4m3 weights: quantize_fp8 / Fp8Tensor::dequantize / Fp8Linear::forward
    //    (crates/sketchpad-core/src/quantization.rs:495, :435, :601), GLU and RoPE epilogues
    pub fn sp_fp8_quantize(
        w: *const c_float, n: i64, k: i64, scale_mode: c_int, w_e4m3: *mut c_void,
        scale: *mut c_float, stream: *mut c_void
    ) -> c_int;
    pub fn sp_fp8_dequant(
        w_e4m3: *const c_void, scale: *const c_float, nscale: i64, n: i64, k: i64,
        out: *mut c_void, out_dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_fp8_linear(
        x: *const c_void, w_e4m3: *const c_void, scale: *const c_float, nscale: i64,
        bias: *const c_void, y: *mut c_void, m: i64, n: i64, k: i64, dtype: c_int,
        stream: *mut c_void
    ) -> c_int;
    pub fn sp_fp8_linear_gated(
        x: *const c_void, w_e4m3: *const c_void, scale: *const c_float, nscale: i64,
        bias: *const c_void, gate: *const c_void, residual: *const c_void, y: *mut c_void,
        m: i64, n: i64, k: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_q8_0_linear_glu(
        x: *const c_void, q: *const c_void, scale: *const c_void, bias: *const c_void,
        y: *mut c_void, m: i64, n: i64, k: i64, glu_kind: c_int, dtype: c_int,
        stream: *mut c_void
    ) -> c_int;
    pub fn sp_fp8_linear_glu(
        x: *const c_void, w_e4m3: *const c_void, scale: *const c_float, nscale: i64,
        bias: *const c_void, y: *mut c_void, m: i64, n: i64, k: i64, glu_kind: c_int,
        dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_q8_0_linear_rope(
        x: *const c_void, q: *const c_void, scale: *const c_void, bias: *const c_void,
        y: *mut c_void, ldy: i64, m: i64, n: i64, k: i64, rope_cos_sin: *const c_float,
        rope_positions: i64, rope_cols: i64, head_dim: i64, pos_offset: i64, pos_div: i64,
        pos_mod: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_fp8_linear_rope(
        x: *const c_void, w_e4m3: *const c_void, scale: *const c_float, nscale: i64,
        bias: *const c_void, y: *mut c_void, ldy: i64, m: i64, n: i64, k: i64,
        rope_cos_sin: *const c_float, rope_positions: i64, rope_cols: i64, head_dim: i64,
        pos_offset: i64, pos_div: i64, pos_mod: i64, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    // -- LayerNorm (crates/sketchpad-core/src/layernorm.rs:63-73: unbiased variance)
    pub fn sp_layernorm(
        x: *const c_void, gamma: *const c_void, beta: *const c_void, y: *mut c_void, rows: i64,
        n: i64, eps: c_float, unbiased: c_int, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_layernorm_add(
        x: *const c_void, x_add: *const c_void, gamma: *const c_void, beta: *const c_void,
        y: *mut c_void, rows: i64, n: i64, eps: c_float, unbiased: c_int, dtype: c_int,
        stream: *mut c_void
    ) -> c_int;
    pub fn sp_layernorm_modulate(
        x: *const c_void, scale: *const c_void, shift: *const c_void, y: *mut c_void,
        rows: i64, n: i64, rows_per_group: i64, mod_stride: i64, eps: c_float, unbiased: c_int,
        dtype: c_int, stream: *mut c_void
    ) -> c_int;
    // -- sampler steps on the device (crates/sketchpad-samplers/src/ddim.rs:157, dpm.rs:101-171)
    pub fn sp_cfg_ddim_step(
        x: *const c_void, eps_uncond: *const c_void, eps_cond: *const c_void,
        noise: *const c_void, out: *mut c_void, n: i64, guidance: c_float,
        sqrt_one_minus_at: c_float, sqrt_at: c_float, sqrt_at_prev: c_float, dir_xt: c_float,
        sigma: c_float, dtype: c_int, stream: *mut c_void
    ) -> c_int;
    pub fn sp_cfg_dpmpp_2m_step(
        x: *const c_void, eps_uncond: *const c_void, eps_cond: *const c_void,
        prev_denoised: *mut c_float, out: *mut c_void, n: i64, guidance: c_float,
        sigma: c_float, sigma_ratio: c_float, one_minus_exp_neg_h: c_float,
        one_plus_coeff: c_float, coeff: c_float, second_order: c_int, dtype: c_int,
        stream: *mut c_void
    ) -> c_int;
    // -- sequence-parallel (Ulysses) exchange over the library's NCCL communicator
    pub fn sp_nccl_unique_id_bytes() -> usize;
    pub fn sp_nccl_unique_id(id_out: *mut c_void, id_bytes: usize) -> c_int;
    pub fn sp_nccl_comm_init(
        comm_out: *mut *mut c_void, nranks: c_int, rank: c_int, id: *const c_void,
        timeout_s: c_double
    ) -> c_int;
    pub fn sp_nccl_comm_poll(comm: *mut c_void, nccl_status_out: *mut c_int) -> c_int;
    pub fn sp_nccl_wait(comm: *mut c_void, stream: *mut c_void, timeout_s: c_double) -> c_int;
    pub fn sp_nccl_comm_abort(comm: *mut c_void) -> c_int;
    pub fn sp_nccl_comm_destroy(comm: *mut c_void, timeout_s: c_double) -> c_int;
    pub fn sp_ulysses_a2a(
        send: *const c_void, recv: *mut c_void, count: i64, dtype: c_int, comm: *mut c_void,
        stream: *mut c_void, timeout_s: c_double
    ) -> c_int;
    pub fn sp_nccl_all_gather(
        send: *const c_void, recv: *mut c_void, count: i64, dtype: c_int, comm: *mut c_void,
        stream: *mut c_void, timeout_s: c_double
    ) -> c_int;
    // -- weight files: GGUF v3 (crates/sketchpad-convert/src/gguf.rs:351-470) and
    //    safetensors (crates/sketchpad-convert/src/loader.rs:60-90), host only
    pub fn sp_model_open(path: *const c_char, file_out: *mut *mut c_void) -> c_int;
    pub fn sp_model_close(file: *mut c_void) -> c_int;
    pub fn sp_model_info(
        file: *mut c_void, container_out: *mut c_int, tensor_count_out: *mut i64,
        meta_count_out: *mut i64
    ) -> c_int;
    pub fn sp_model_meta_key(
        file: *mut c_void, index: i64, name_out: *mut c_char, name_cap: usize
    ) -> c_int;
    pub fn sp_model_tensor_info(
        file: *mut c_void, index: i64, name_out: *mut c_char, name_cap: usize,
        type_out: *mut c_int, ndims_out: *mut c_int, dims_out: *mut i64, nbytes_out: *mut u64
    ) -> c_int;
    pub fn sp_model_find(file: *mut c_void, name: *const c_char, index_out: *mut i64) -> c_int;
    pub fn sp_model_tensor_data(
        file: *mut c_void, index: i64, data_out: *mut *const u8
    ) -> c_int;

}
