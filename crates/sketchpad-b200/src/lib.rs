//! sketchpad-b200: the reference's GPU operator surface (crates/sketchpad-cubecl) over the
//! sm_100a kernels of libsketchpad_b200, so UNet / DiT / sampler code keeps its calls:
//!
//! | reference (crates/sketchpad-cubecl/src)                        | here                      |
//! |----------------------------------------------------------------|---------------------------|
//! | `attention.rs:40-68` `FlashAttentionOptions`                     | [`FlashAttentionOptions`] |
//! | `attention.rs:97` `flash_attention`                              | [`flash_attention`]       |
//! | `attention.rs:119` `flash_attention_masked`                      | [`flash_attention_masked`]|
//! | `groupnorm_silu.rs:22-46` `GroupNormSiLuOptions`                 | [`GroupNormSiLuOptions`]  |
//! | `groupnorm_silu.rs:232` `groupnorm_silu`, `:323` `groupnorm`     | [`groupnorm_silu`], [`groupnorm`] |
//! | `quantized_matmul.rs:376` `dequantize_q8_0`                      | [`dequantize_q8_0`]       |
//! | `quantized_matmul.rs:655-767` `GpuQuantizedLinear`               | [`GpuQuantizedLinear`]    |
//! | `sketchpad-core/src/quantization.rs:422-615` FP8                 | [`quantize_fp8`], [`Fp8Tensor`], [`Fp8Linear`] |
//!
//! As in the reference, inputs are taken by value (a [`CubeTensor`] is a cheap handle) and
//! each operator returns a tensor it allocated; launches are asynchronous on the tensor's
//! [`ComputeClient`] stream.  Errors follow the reference: attention returns
//! `Err(AttentionSetupError)`, GroupNorm and the quantized layers panic on bad shapes.
//! [`UlyssesComm`] is the sequence-parallel exchange the reference does not have.
use core::ffi::{c_int, c_void, CStr};
use std::sync::Arc;

use sketchpad_b200_sys as sys;

// ------------------------------------------------------------------------------------------
// CUDA runtime: the allocation and copy calls the reference's ComputeClient makes
// ------------------------------------------------------------------------------------------
#[link(name = "cudart")]
extern "C" {
    fn cudaMallocAsync(ptr: *mut *mut c_void, bytes: usize, stream: *mut c_void) -> c_int;
    fn cudaFreeAsync(ptr: *mut c_void, stream: *mut c_void) -> c_int;
    fn cudaMemcpyAsync(dst: *mut c_void, src: *const c_void, bytes: usize, kind: c_int,
                       stream: *mut c_void) -> c_int;
    fn cudaStreamSynchronize(stream: *mut c_void) -> c_int;
}
const H2D: c_int = 1;
const D2H: c_int = 2;

/// A failed library call: the status (`SP_ERR_*`) and the library's message.
#[derive(Debug, Clone)]
pub struct SketchpadError {
    pub status: c_int,
    pub message: String,
}

impl std::fmt::Display for SketchpadError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "{} (status {})", self.message, self.status)
    }
}
impl std::error::Error for SketchpadError {}

/// Where the reference returns `Err(AttentionSetupError)` (attention.rs:97-104).
#[derive(Debug, Clone)]
pub struct AttentionSetupError(pub String);

impl std::fmt::Display for AttentionSetupError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        f.write_str(&self.0)
    }
}
impl std::error::Error for AttentionSetupError {}

fn last_error() -> String {
    // SAFETY: sp_last_error returns a NUL-terminated thread-local string
    unsafe { CStr::from_ptr(sys::sp_last_error()) }.to_string_lossy().into_owned()
}

fn check(rc: c_int) -> Result<(), SketchpadError> {
    if rc == sys::SP_OK {
        Ok(())
    } else {
        Err(SketchpadError { status: rc, message: last_error() })
    }
}

#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum DType {
    F32,
    F16,
    BF16,
}

impl DType {
    pub fn code(self) -> c_int {
        match self {
            DType::F32 => sys::SP_F32,
            DType::F16 => sys::SP_F16,
            DType::BF16 => sys::SP_BF16,
        }
    }
    pub fn size(self) -> usize {
        if self == DType::F32 { 4 } else { 2 }
    }
}

/// The stream every launch and allocation of a tensor is ordered on (the reference's
/// `ComputeClient`, one queue per device).  The null stream is CUDA's legacy default.
#[derive(Clone, Copy, Debug)]
pub struct ComputeClient {
    stream: *mut c_void,
}
// SAFETY: a cudaStream_t may be used from any host thread
unsafe impl Send for ComputeClient {}
unsafe impl Sync for ComputeClient {}

impl ComputeClient {
    /// # Safety
    /// `stream` must be a live `cudaStream_t` of the current device (or null).
    pub unsafe fn from_stream(stream: *mut c_void) -> Self {
        ComputeClient { stream }
    }
    pub fn default_stream() -> Self {
        ComputeClient { stream: core::ptr::null_mut() }
    }
    pub fn stream(&self) -> *mut c_void {
        self.stream
    }
    fn alloc(&self, bytes: usize) -> Arc<Buffer> {
        let mut ptr = core::ptr::null_mut();
        // SAFETY: plain stream-ordered allocation
        let rc = unsafe { cudaMallocAsync(&mut ptr, bytes.max(1), self.stream) };
        assert!(rc == 0, "cudaMallocAsync of {bytes} bytes failed ({rc})");
        Arc::new(Buffer { ptr, stream: self.stream })
    }
    /// Copies host bytes into a new device buffer; complete when this returns.
    fn upload(&self, host: &[u8]) -> Arc<Buffer> {
        let b = self.alloc(host.len());
        // SAFETY: b holds host.len() bytes; the copy is waited for before `host` can go away
        let rc = unsafe {
            cudaMemcpyAsync(b.ptr, host.as_ptr().cast(), host.len(), H2D, self.stream)
                | cudaStreamSynchronize(self.stream)
        };
        assert!(rc == 0, "upload of {} bytes failed", host.len());
        b
    }
    /// `into_data()`: waits for the stream and copies a tensor's memory to the host.
    pub fn read(&self, t: &CubeTensor) -> Vec<u8> {
        assert!(t.is_contiguous(), "read needs a contiguous tensor");
        let n = t.numel() * t.dtype.size();
        let mut host = vec![0u8; n];
        // SAFETY: t spans n bytes of device memory
        let rc = unsafe {
            cudaMemcpyAsync(host.as_mut_ptr().cast(), t.ptr, n, D2H, self.stream)
                | cudaStreamSynchronize(self.stream)
        };
        assert!(rc == 0, "read of {n} bytes failed");
        host
    }
}

struct Buffer {
    ptr: *mut c_void,
    stream: *mut c_void,
}
unsafe impl Send for Buffer {}
unsafe impl Sync for Buffer {}
impl Drop for Buffer {
    fn drop(&mut self) {
        // SAFETY: freed in stream order after every launch that used it
        unsafe { cudaFreeAsync(self.ptr, self.stream) };
    }
}

/// A strided device tensor: shape in the reference's dimension order, strides in elements.
/// Owns its memory when an operator allocated it; wraps caller memory via `from_raw`.
#[derive(Clone)]
pub struct CubeTensor {
    pub client: ComputeClient,
    pub ptr: *mut c_void,
    pub shape: Vec<usize>,
    pub strides: Vec<usize>,
    pub dtype: DType,
    _owner: Option<Arc<Buffer>>,
}

impl CubeTensor {
    /// # Safety
    /// `ptr` must address device memory covering every element the shape and strides
    /// reach, alive for as long as the tensor is used.
    pub unsafe fn from_raw(client: ComputeClient, ptr: *mut c_void, shape: Vec<usize>,
                           strides: Vec<usize>, dtype: DType) -> Self {
        assert_eq!(shape.len(), strides.len(), "one stride per dimension");
        CubeTensor { client, ptr, shape, strides, dtype, _owner: None }
    }
    /// A new contiguous tensor (`empty_device_dtype`).
    pub fn empty(client: &ComputeClient, shape: Vec<usize>, dtype: DType) -> Self {
        let n: usize = shape.iter().product();
        let buf = client.alloc(n * dtype.size());
        let strides = contiguous_strides(&shape);
        CubeTensor { client: *client, ptr: buf.ptr, shape, strides, dtype, _owner: Some(buf) }
    }
    /// A contiguous tensor with these host bytes.
    pub fn from_bytes(client: &ComputeClient, bytes: &[u8], shape: Vec<usize>, dtype: DType) -> Self {
        assert_eq!(bytes.len(), shape.iter().product::<usize>() * dtype.size());
        let buf = client.upload(bytes);
        let strides = contiguous_strides(&shape);
        CubeTensor { client: *client, ptr: buf.ptr, shape, strides, dtype, _owner: Some(buf) }
    }
    pub fn numel(&self) -> usize {
        self.shape.iter().product()
    }
    pub fn is_contiguous(&self) -> bool {
        self.strides == contiguous_strides(&self.shape)
            || self.shape.iter().zip(&self.strides).zip(contiguous_strides(&self.shape))
                .all(|((&d, &s), c)| d <= 1 || s == c)
    }
    fn strides_i64(&self) -> Vec<i64> {
        self.strides.iter().map(|&s| s as i64).collect()
    }
}

fn contiguous_strides(shape: &[usize]) -> Vec<usize> {
    let mut s = vec![1usize; shape.len()];
    for i in (0..shape.len().saturating_sub(1)).rev() {
        s[i] = s[i + 1] * shape[i + 1];
    }
    s
}

// ------------------------------------------------------------------------------------------
// Flash attention (attention.rs:40-178)
// ------------------------------------------------------------------------------------------
/// Options for flash attention (attention.rs:40-68).
#[derive(Debug, Clone, Default)]
pub struct FlashAttentionOptions {
    /// Output dtype; `None` uses the query dtype.
    pub out_dtype: Option<DType>,
    /// Exclude keys after the query position.
    pub causal: bool,
}

impl FlashAttentionOptions {
    pub fn causal() -> Self {
        FlashAttentionOptions { out_dtype: None, causal: true }
    }
    pub fn with_dtype(mut self, dtype: DType) -> Self {
        self.out_dtype = Some(dtype);
        self
    }
    pub fn with_causal(mut self, causal: bool) -> Self {
        self.causal = causal;
        self
    }
}

/// softmax(Q K^T / sqrt(d) [causal]) V -> [batch, heads, seq_q, val_dim] (attention.rs:97).
/// bf16 or f16 query/key/value with any strides (innermost stride 1); f32 accumulate.
pub fn flash_attention(query: CubeTensor, key: CubeTensor, value: CubeTensor,
                       options: FlashAttentionOptions) -> Result<CubeTensor, AttentionSetupError> {
    flash_attention_impl(query, key, value, None, options)
}

/// The same with an additive f32 [seq_q, seq_k] mask (attention.rs:119).
pub fn flash_attention_masked(query: CubeTensor, key: CubeTensor, value: CubeTensor,
                              mask: CubeTensor, options: FlashAttentionOptions)
                              -> Result<CubeTensor, AttentionSetupError> {
    flash_attention_impl(query, key, value, Some(mask), options)
}

fn flash_attention_impl(q: CubeTensor, k: CubeTensor, v: CubeTensor, mask: Option<CubeTensor>,
                        options: FlashAttentionOptions) -> Result<CubeTensor, AttentionSetupError> {
    let setup = |m: &str| Err(AttentionSetupError(m.to_string()));
    if q.shape.len() != 4 || k.shape.len() != 4 || v.shape.len() != 4 {
        return setup("query, key and value must be [batch, heads, seq, dim]");
    }
    let (b, h, sq, d) = (q.shape[0], q.shape[1], q.shape[2], q.shape[3]);
    let (skv, dv) = (k.shape[2], v.shape[3]);
    if k.shape[0] != b || k.shape[1] != h || k.shape[3] != d || v.shape[0] != b
        || v.shape[1] != h || v.shape[2] != skv {
        return setup("query, key and value shapes do not match");
    }
    if q.dtype != k.dtype || q.dtype != v.dtype || q.dtype == DType::F32 {
        return setup("query, key and value must share one dtype, bf16 or f16");
    }
    let (mptr, mstride) = match &mask {
        None => (core::ptr::null(), 0i64),
        Some(m) => {
            if m.shape != [sq, skv] || m.dtype != DType::F32 || m.strides[1] != 1 {
                return setup("mask must be an f32 [seq_q, seq_k] tensor with unit column stride");
            }
            (m.ptr as *const f32, m.strides[0] as i64)
        }
    };
    let od = options.out_dtype.unwrap_or(q.dtype);
    let out = CubeTensor::empty(&q.client, vec![b, h, sq, dv], od);
    let (qs, ks, vs, os) = (q.strides_i64(), k.strides_i64(), v.strides_i64(), out.strides_i64());
    // SAFETY: every pointer spans its tensor; strides have 4 entries each
    let rc = unsafe {
        sys::sp_flash_attn_fwd(q.ptr, k.ptr, v.ptr, mptr, mstride, out.ptr, b as i64, h as i64,
                               sq as i64, skv as i64, d as i64, dv as i64, qs.as_ptr(),
                               ks.as_ptr(), vs.as_ptr(), os.as_ptr(), q.dtype.code(), od.code(),
                               options.causal as c_int, 0.0, q.client.stream())
    };
    match rc {
        sys::SP_OK => Ok(out),
        sys::SP_ERR_INVALID_ARG | sys::SP_ERR_SHAPE | sys::SP_ERR_DTYPE | sys::SP_ERR_ALIGN => {
            Err(AttentionSetupError(last_error()))
        }
        _ => panic!("flash attention: {}", last_error()),
    }
}

// ------------------------------------------------------------------------------------------
// GroupNorm (+ SiLU) (groupnorm_silu.rs:22-46, :232, :323)
// ------------------------------------------------------------------------------------------
/// Options for GroupNorm + SiLU (groupnorm_silu.rs:22-46).
#[derive(Debug, Clone, Copy)]
pub struct GroupNormSiLuOptions {
    pub num_groups: usize,
    pub eps: f32,
}

impl Default for GroupNormSiLuOptions {
    fn default() -> Self {
        GroupNormSiLuOptions { num_groups: 32, eps: 1e-5 }
    }
}

impl GroupNormSiLuOptions {
    pub fn with_groups(num_groups: usize) -> Self {
        GroupNormSiLuOptions { num_groups, eps: 1e-5 }
    }
}

fn groupnorm_act(input: CubeTensor, weight: CubeTensor, bias: CubeTensor,
                 options: GroupNormSiLuOptions, act: c_int) -> CubeTensor {
    assert_eq!(input.shape.len(), 4, "groupnorm: input must be [batch, channels, height, width]");
    let (b, c, h, w) = (input.shape[0], input.shape[1], input.shape[2], input.shape[3]);
    // the reference panics here too (groupnorm_silu.rs:240-245)
    assert!(options.num_groups > 0 && c % options.num_groups == 0,
            "channels ({c}) must be divisible by num_groups ({})", options.num_groups);
    assert!(weight.numel() == c && bias.numel() == c && weight.dtype == input.dtype
            && bias.dtype == input.dtype, "weight and bias must be [channels] of the input dtype");
    let xs = input.strides_i64();
    let mut ys = [0i64; 4];
    let g = options.num_groups as i64;
    // SAFETY: xs has 4 entries; ys receives 4
    check(unsafe {
        sys::sp_groupnorm_act_output_strides(b as i64, c as i64, h as i64, w as i64, xs.as_ptr(),
                                             ys.as_mut_ptr())
    }).expect("groupnorm output layout");
    let mut out = CubeTensor::empty(&input.client, vec![b, c, h, w], input.dtype);
    out.strides = ys.iter().map(|&s| s as usize).collect();
    let ws_bytes = unsafe {
        sys::sp_groupnorm_act_workspace_size(b as i64, c as i64, h as i64, w as i64, xs.as_ptr(),
                                             g, input.dtype.code())
    };
    let ws = if ws_bytes > 0 { Some(input.client.alloc(ws_bytes)) } else { None };
    let wsp = ws.as_ref().map_or(core::ptr::null_mut(), |b| b.ptr);
    // SAFETY: pointers span their tensors; the workspace lives until after the launch is
    // ordered (freed in stream order when `ws` drops)
    check(unsafe {
        sys::sp_groupnorm_act(input.ptr, weight.ptr, bias.ptr, out.ptr, b as i64, c as i64,
                              h as i64, w as i64, xs.as_ptr(), g, options.eps, act,
                              input.dtype.code(), wsp, ws_bytes, input.client.stream())
    }).unwrap_or_else(|e| panic!("groupnorm: {e}"));
    out
}

/// GroupNorm followed by SiLU (groupnorm_silu.rs:232).  The output keeps a dense
/// channels-last input's layout, else it is contiguous NCHW.
pub fn groupnorm_silu(input: CubeTensor, weight: CubeTensor, bias: CubeTensor,
                      options: GroupNormSiLuOptions) -> CubeTensor {
    groupnorm_act(input, weight, bias, options, sys::SP_ACT_SILU)
}

/// GroupNorm alone (groupnorm_silu.rs:323).
pub fn groupnorm(input: CubeTensor, weight: CubeTensor, bias: CubeTensor,
                 options: GroupNormSiLuOptions) -> CubeTensor {
    groupnorm_act(input, weight, bias, options, sys::SP_ACT_NONE)
}

// ------------------------------------------------------------------------------------------
// Quantized linears (quantized_matmul.rs:33-43, :376-408, :655-767)
// ------------------------------------------------------------------------------------------
/// GGUF quantization formats with a fused GPU path (quantized_matmul.rs:33-43).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum GpuQuantType {
    Q8_0,
    Q4K,
    Q2K,
    Q3K,
}

impl GpuQuantType {
    fn kquant_fmt(self) -> c_int {
        match self {
            GpuQuantType::Q4K => sys::SP_QK_Q4_K,
            GpuQuantType::Q2K => sys::SP_QK_Q2_K,
            GpuQuantType::Q3K => sys::SP_QK_Q3_K,
            GpuQuantType::Q8_0 => unreachable!(),
        }
    }
    fn sub_block(self) -> usize {
        if self == GpuQuantType::Q4K { 32 } else { 16 }
    }
}

/// A linear projection whose weights stay quantized in device memory; `forward` decodes them
/// inside the GEMM mainloop (no dequantized copy is ever written).
pub struct GpuQuantizedLinear {
    client: ComputeClient,
    quant_type: GpuQuantType,
    out_features: usize,
    in_features: usize,
    q: Arc<Buffer>,
    a: Arc<Buffer>,
    b: Option<Arc<Buffer>>,
    bias: Option<CubeTensor>,
}

fn as_bytes<T: Copy>(v: &[T]) -> &[u8] {
    // SAFETY: plain-old-data slice viewed as bytes
    unsafe { core::slice::from_raw_parts(v.as_ptr().cast(), core::mem::size_of_val(v)) }
}

impl GpuQuantizedLinear {
    /// `GpuQuantizedLinear::from_bytes` (quantized_matmul.rs:670-702): raw GGUF blocks on the
    /// host, repacked losslessly into the planar layout the fused GEMM reads.  `dtype` is the
    /// activation dtype of `forward` (bf16).
    pub fn from_bytes(bytes: &[u8], quant_type: GpuQuantType, out_features: usize,
                      in_features: usize, client: &ComputeClient, dtype: DType) -> Self {
        assert_eq!(dtype, DType::BF16, "the fused GEMM takes bf16 activations");
        let (n, k) = (out_features, in_features);
        let (q, a, b) = match quant_type {
            GpuQuantType::Q8_0 => {
                let mut q = vec![0i8; n * k];
                let mut sc = vec![0u16; n * (k / 32)];
                // SAFETY: q and sc have the sizes the header gives
                check(unsafe {
                    sys::sp_q8_0_repack_host(bytes.as_ptr(), bytes.len(), n as i64, k as i64,
                                             q.as_mut_ptr(), sc.as_mut_ptr())
                }).unwrap_or_else(|e| panic!("Q8_0 repack: {e}"));
                (client.upload(as_bytes(&q)), client.upload(as_bytes(&sc)), None)
            }
            kq => {
                let sub = kq.sub_block();
                let mut q = vec![0u8; n * k / 2];
                let mut fa = vec![0f32; n * (k / sub)];
                let mut fb = vec![0f32; n * (k / sub)];
                check(unsafe {
                    sys::sp_kquant_repack_host(kq.kquant_fmt(), bytes.as_ptr(), bytes.len(),
                                               n as i64, k as i64, q.as_mut_ptr(),
                                               fa.as_mut_ptr(), fb.as_mut_ptr())
                }).unwrap_or_else(|e| panic!("K-quant repack: {e}"));
                (client.upload(&q), client.upload(as_bytes(&fa)), Some(client.upload(as_bytes(&fb))))
            }
        };
        GpuQuantizedLinear { client: *client, quant_type, out_features, in_features, q, a, b,
                             bias: None }
    }

    /// Adds a bf16 [out_features] bias to `forward`.
    pub fn with_bias(mut self, bias: CubeTensor) -> Self {
        assert!(bias.numel() == self.out_features && bias.dtype == DType::BF16);
        self.bias = Some(bias);
        self
    }

    /// `dequantize` (quantized_matmul.rs:705): [out_features, in_features] f32, bit-exact
    /// with the reference's CPU decode.
    pub fn dequantize(&self) -> CubeTensor {
        let out = CubeTensor::empty(&self.client, vec![self.out_features, self.in_features],
                                    DType::F32);
        let (n, k) = (self.out_features as i64, self.in_features as i64);
        let rc = unsafe {
            match self.quant_type {
                GpuQuantType::Q8_0 => sys::sp_q8_0_dequant(self.q.ptr, self.a.ptr, n, k, out.ptr,
                                                           sys::SP_F32, self.client.stream()),
                kq => sys::sp_kquant_dequant(kq.kquant_fmt(), self.q.ptr, self.a.ptr.cast(),
                                             self.b.as_ref().unwrap().ptr.cast(), n, k, out.ptr,
                                             sys::SP_F32, self.client.stream()),
            }
        };
        check(rc).unwrap_or_else(|e| panic!("dequantize: {e}"));
        out
    }

    /// `forward` (quantized_matmul.rs:752-766): input [..., in_features] bf16, contiguous ->
    /// [..., out_features] bf16 = input . dequant(W)^T (+ bias).
    pub fn forward(&self, input: CubeTensor) -> CubeTensor {
        assert!(input.dtype == DType::BF16 && input.is_contiguous()
                && input.shape.last() == Some(&self.in_features),
                "forward: input must be contiguous bf16 [..., in_features]");
        let m = (input.numel() / self.in_features) as i64;
        let mut shape = input.shape.clone();
        *shape.last_mut().unwrap() = self.out_features;
        let out = CubeTensor::empty(&self.client, shape, DType::BF16);
        let bias = self.bias.as_ref().map_or(core::ptr::null(), |b| b.ptr as *const c_void);
        let (n, k) = (self.out_features as i64, self.in_features as i64);
        let rc = unsafe {
            match self.quant_type {
                GpuQuantType::Q8_0 => sys::sp_q8_0_linear(input.ptr, self.q.ptr, self.a.ptr, bias,
                                                          out.ptr, m, n, k, sys::SP_BF16,
                                                          self.client.stream()),
                kq => sys::sp_kquant_linear(kq.kquant_fmt(), input.ptr, self.q.ptr,
                                            self.a.ptr.cast(),
                                            self.b.as_ref().unwrap().ptr.cast(), bias, out.ptr,
                                            m, n, k, sys::SP_BF16, self.client.stream()),
            }
        };
        check(rc).unwrap_or_else(|e| panic!("quantized linear: {e}"));
        out
    }

    pub fn out_features(&self) -> usize {
        self.out_features
    }
    pub fn in_features(&self) -> usize {
        self.in_features
    }
}

/// `dequantize_q8_0` (quantized_matmul.rs:376-408): GGUF Q8_0 bytes -> [out_f, in_f] f32.
pub fn dequantize_q8_0(bytes: &[u8], out_f: usize, in_f: usize, client: &ComputeClient) -> CubeTensor {
    GpuQuantizedLinear::from_bytes(bytes, GpuQuantType::Q8_0, out_f, in_f, client, DType::BF16)
        .dequantize()
}

// ------------------------------------------------------------------------------------------
// FP8 e4m3 weights (sketchpad-core/src/quantization.rs:422-615)
// ------------------------------------------------------------------------------------------
/// e4m3 bytes [N, K] + f32 scales (one per output channel, or one).
pub struct Fp8Tensor {
    client: ComputeClient,
    data: Arc<Buffer>,
    scale: Arc<Buffer>,
    nscale: usize,
    pub shape: [usize; 2],
}

/// `quantize_fp8` with the E4M3 config (quantization.rs:495-577) of an f32 [N, K] tensor.
pub fn quantize_fp8(tensor: &CubeTensor, per_channel: bool) -> Fp8Tensor {
    assert!(tensor.shape.len() == 2 && tensor.dtype == DType::F32 && tensor.is_contiguous(),
            "quantize_fp8: weights must be contiguous f32 [out, in]");
    let (n, k) = (tensor.shape[0], tensor.shape[1]);
    let nscale = if per_channel { n } else { 1 };
    let data = tensor.client.alloc(n * k);
    let scale = tensor.client.alloc(nscale * 4);
    let mode = if per_channel { sys::SP_FP8_PER_CHANNEL } else { sys::SP_FP8_PER_TENSOR };
    check(unsafe {
        sys::sp_fp8_quantize(tensor.ptr as *const f32, n as i64, k as i64, mode, data.ptr,
                             scale.ptr.cast(), tensor.client.stream())
    }).unwrap_or_else(|e| panic!("quantize_fp8: {e}"));
    Fp8Tensor { client: tensor.client, data, scale, nscale, shape: [n, k] }
}

impl Fp8Tensor {
    /// `Fp8Tensor::dequantize` (quantization.rs:435-447): data * scale[row] in f32.
    pub fn dequantize(&self) -> CubeTensor {
        let out = CubeTensor::empty(&self.client, self.shape.to_vec(), DType::F32);
        check(unsafe {
            sys::sp_fp8_dequant(self.data.ptr, self.scale.ptr.cast(), self.nscale as i64,
                                self.shape[0] as i64, self.shape[1] as i64, out.ptr, sys::SP_F32,
                                self.client.stream())
        }).unwrap_or_else(|e| panic!("fp8 dequantize: {e}"));
        out
    }
}

/// `Fp8Linear` (quantization.rs:587-615): y = x . dequant(W)^T + b, the e4m3 decode inside
/// the GEMM and the scale in its epilogue.
pub struct Fp8Linear {
    weight: Fp8Tensor,
    bias: Option<CubeTensor>,
}

impl Fp8Linear {
    pub fn new(weight: Fp8Tensor, bias: Option<CubeTensor>) -> Self {
        if let Some(b) = &bias {
            assert!(b.numel() == weight.shape[0] && b.dtype == DType::BF16,
                    "Fp8Linear: bias must be [out_features] bf16");
        }
        Fp8Linear { weight, bias }
    }
    pub fn forward(&self, x: CubeTensor) -> CubeTensor {
        let [n, k] = self.weight.shape;
        assert!(x.dtype == DType::BF16 && x.is_contiguous() && x.shape.last() == Some(&k),
                "Fp8Linear::forward: x must be contiguous bf16 [..., in_features]");
        let mut shape = x.shape.clone();
        *shape.last_mut().unwrap() = n;
        let out = CubeTensor::empty(&x.client, shape, DType::BF16);
        let bias = self.bias.as_ref().map_or(core::ptr::null(), |b| b.ptr as *const c_void);
        check(unsafe {
            sys::sp_fp8_linear(x.ptr, self.weight.data.ptr, self.weight.scale.ptr.cast(),
                               self.weight.nscale as i64, bias, out.ptr,
                               (x.numel() / k) as i64, n as i64, k as i64, sys::SP_BF16,
                               x.client.stream())
        }).unwrap_or_else(|e| panic!("fp8 linear: {e}"));
        out
    }
}

// ------------------------------------------------------------------------------------------
// Sequence-parallel exchange (no reference counterpart: the reference runs on one device)
// ------------------------------------------------------------------------------------------
/// The library's non-blocking NCCL communicator for the Ulysses all-to-all around each Wan
/// self-attention.  Every call is bounded by `timeout_s`; on an NCCL error or an expired
/// deadline the communicator is aborted and the call returns `SP_ERR_COMM`.
pub struct UlyssesComm {
    comm: *mut c_void,
    pub rank: usize,
    pub size: usize,
    pub timeout_s: f64,
}
unsafe impl Send for UlyssesComm {}

impl UlyssesComm {
    /// A fresh NCCL unique id; one rank makes it and sends it to the others.
    pub fn unique_id() -> Result<Vec<u8>, SketchpadError> {
        let n = unsafe { sys::sp_nccl_unique_id_bytes() };
        let mut id = vec![0u8; n];
        check(unsafe { sys::sp_nccl_unique_id(id.as_mut_ptr().cast(), n) })?;
        Ok(id)
    }
    /// Joins rank `rank` of `size` on the current device.
    pub fn new(rank: usize, size: usize, id: &[u8], timeout_s: f64) -> Result<Self, SketchpadError> {
        let mut comm = core::ptr::null_mut();
        check(unsafe {
            sys::sp_nccl_comm_init(&mut comm, size as c_int, rank as c_int, id.as_ptr().cast(),
                                   timeout_s)
        })?;
        Ok(UlyssesComm { comm, rank, size, timeout_s })
    }
    /// sp_ulysses_a2a: chunk p of `send` (numel / size elements) goes to rank p, chunk p of
    /// `recv` comes from rank p.  Both contiguous, same dtype and size.
    pub fn all_to_all(&self, send: &CubeTensor, recv: &CubeTensor) -> Result<(), SketchpadError> {
        assert!(send.numel() == recv.numel() && send.numel() % self.size == 0
                && send.dtype == recv.dtype && send.is_contiguous() && recv.is_contiguous());
        check(unsafe {
            sys::sp_ulysses_a2a(send.ptr, recv.ptr, (send.numel() / self.size) as i64,
                                send.dtype.code(), self.comm, send.client.stream(), self.timeout_s)
        })
    }
    /// Waits for `client`'s stream while watching the communicator (abort on failure).
    pub fn wait(&self, client: &ComputeClient) -> Result<(), SketchpadError> {
        check(unsafe { sys::sp_nccl_wait(self.comm, client.stream(), self.timeout_s) })
    }
    pub fn abort(mut self) {
        unsafe { sys::sp_nccl_comm_abort(self.comm) };
        self.comm = core::ptr::null_mut();
    }
}

impl Drop for UlyssesComm {
    fn drop(&mut self) {
        if !self.comm.is_null() {
            unsafe { sys::sp_nccl_comm_destroy(self.comm, self.timeout_s) };
        }
    }
}

// ------------------------------------------------------------------------------------------
// Weight files (crates/sketchpad-convert/src/gguf.rs:351-470, loader.rs:60-90)
// ------------------------------------------------------------------------------------------
/// One tensor of a GGUF or safetensors file: `sp_tensor_type`, row-major shape, byte size.
#[derive(Debug, Clone)]
pub struct TensorInfo {
    pub name: String,
    pub type_code: c_int,
    pub shape: Vec<usize>,
    pub nbytes: usize,
    index: i64,
}

/// A GGUF v3 or safetensors file, memory-mapped by the library (host only).
pub struct ModelFile {
    handle: *mut c_void,
    pub container: c_int,
    pub tensors: Vec<TensorInfo>,
}
unsafe impl Send for ModelFile {}

impl ModelFile {
    pub fn open(path: &str) -> Result<Self, SketchpadError> {
        let cpath = std::ffi::CString::new(path).expect("path without NUL");
        let mut handle = core::ptr::null_mut();
        check(unsafe { sys::sp_model_open(cpath.as_ptr(), &mut handle) })?;
        let (mut container, mut nt, mut nm) = (0, 0i64, 0i64);
        let mut file = ModelFile { handle, container: 0, tensors: Vec::new() };
        check(unsafe { sys::sp_model_info(handle, &mut container, &mut nt, &mut nm) })?;
        file.container = container;
        let mut name = vec![0 as core::ffi::c_char; 4096];
        for i in 0..nt {
            let (mut t, mut nd, mut nb) = (0, 0, 0u64);
            let mut dims = [0i64; 8];
            check(unsafe {
                sys::sp_model_tensor_info(handle, i, name.as_mut_ptr(), name.len(), &mut t, &mut nd,
                                          dims.as_mut_ptr(), &mut nb)
            })?;
            let n = unsafe { CStr::from_ptr(name.as_ptr()) }.to_string_lossy().into_owned();
            file.tensors.push(TensorInfo { name: n, type_code: t, index: i, nbytes: nb as usize,
                                           shape: dims[..nd as usize].iter().map(|&d| d as usize).collect() });
        }
        Ok(file)
    }

    pub fn info(&self, name: &str) -> Option<&TensorInfo> {
        self.tensors.iter().find(|t| t.name == name)
    }

    /// The tensor's bytes inside the map (GgufFile::tensor_raw_data, gguf.rs:448-470).
    pub fn raw(&self, info: &TensorInfo) -> &[u8] {
        let mut p: *const u8 = core::ptr::null();
        check(unsafe { sys::sp_model_tensor_data(self.handle, info.index, &mut p) })
            .expect("tensor data");
        // SAFETY: the library maps nbytes at p for as long as the file is open
        unsafe { core::slice::from_raw_parts(p, info.nbytes) }
    }

    /// A GpuQuantizedLinear over a 2-D GGUF Q8_0 / Q4_K / Q2_K / Q3_K weight.
    pub fn quantized_linear(&self, name: &str, client: &ComputeClient) -> GpuQuantizedLinear {
        let info = self.info(name).unwrap_or_else(|| panic!("tensor '{name}' not found"));
        let qt = match info.type_code - sys::SP_T_GGML_BASE {
            8 => GpuQuantType::Q8_0,
            10 => GpuQuantType::Q2K,
            11 => GpuQuantType::Q3K,
            12 => GpuQuantType::Q4K,
            t => panic!("tensor '{name}': ggml type {t} has no fused GPU path"),
        };
        assert_eq!(info.shape.len(), 2, "tensor '{name}' is not 2-D");
        GpuQuantizedLinear::from_bytes(self.raw(info), qt, info.shape[0], info.shape[1], client,
                                       DType::BF16)
    }
}

impl Drop for ModelFile {
    fn drop(&mut self) {
        unsafe { sys::sp_model_close(self.handle) };
    }
}
