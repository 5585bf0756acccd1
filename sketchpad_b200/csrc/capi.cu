// capi.cu -- shared C-ABI plumbing: error strings, device checks, TMA descriptor encoding,
// and the device watchdog word used by the bounded waits in tc.cuh.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "tc.cuh"

namespace sp {

__device__ int g_watchdog = 0;

namespace {
thread_local std::string t_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

void clear_error() { t_last_error.clear(); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return SP_OK;
}

int require_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(SP_ERR_DEVICE, "no CUDA device");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return set_error(SP_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                     dev, major, minor);
  return SP_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev;
}

// The library's stream-ordered scratch pool for this device (split-K partials): freed blocks
// stay in the pool (release threshold = max), so the per-call allocate / free pair is cheap
// after the first call of a size.  Created once per device; null if the pool cannot be made.
cudaMemPool_t scratch_pool() {
  static cudaMemPool_t pools[64] = {};
  static int state[64] = {};  // 0 none, 1 creating, 2 ready, 3 failed
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  int st = __atomic_load_n(&state[dev], __ATOMIC_ACQUIRE);
  if (st == 2) return pools[dev];
  if (st == 3) return nullptr;
  int expected = 0;
  if (__atomic_compare_exchange_n(&state[dev], &expected, 1, false, __ATOMIC_ACQ_REL,
                                  __ATOMIC_ACQUIRE)) {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) == cudaSuccess) {
      uint64_t keep = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      pools[dev] = pool;
      __atomic_store_n(&state[dev], 2, __ATOMIC_RELEASE);
      return pool;
    }
    cudaGetLastError();
    __atomic_store_n(&state[dev], 3, __ATOMIC_RELEASE);
    return nullptr;
  }
  // another thread is creating it: wait (bounded by the creation itself)
  while ((st = __atomic_load_n(&state[dev], __ATOMIC_ACQUIRE)) == 1) {
  }
  return st == 2 ? pools[dev] : nullptr;
}

bool first_time_on_device(unsigned long long* flag_bits) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return true;
  const unsigned long long bit = 1ull << dev;
  const unsigned long long old = __atomic_fetch_or(flag_bits, bit, __ATOMIC_ACQ_REL);
  return (old & bit) == 0;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(SP_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SP_ERR_ALIGN, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return SP_OK;
}

}  // namespace sp

extern "C" {

int sp_abi_version(void) { return SP_ABI_VERSION; }

const char* sp_last_error(void) { return sp::t_last_error.c_str(); }

int sp_watchdog_read_and_clear(void* stream, int* code_out) {
  if (!code_out) return sp::set_error(SP_ERR_INVALID_ARG, "code_out is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int zero = 0, val = 0;
  if (cudaMemcpyFromSymbolAsync(&val, sp::g_watchdog, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaMemcpyToSymbolAsync(sp::g_watchdog, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return sp::set_error(SP_ERR_LAUNCH, "watchdog read failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
  *code_out = val;
  return SP_OK;
}

}  // extern "C"
