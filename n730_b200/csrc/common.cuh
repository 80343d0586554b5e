// Shared definitions for the N730 B200 kernels and C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <mutex>

#define N730_API extern "C" __attribute__((visibility("default")))

// Return codes.  0/-10/-11/-12 keep the reference meanings
// (src-code/cpp/n730_cuda.cu:41-44); the rest are new.
enum : int {
  N730_OK = 0,
  N730_CUDA_ERR = -10,
  N730_OOM = -11,
  N730_NULL = -12,
  N730_BAD_ARG = -13,      // shape / layout / precision not accepted
  N730_UNSUPPORTED = -14,  // valid request this build does not implement
  N730_TIMEOUT = -15,      // a bounded device wait ran out
  N730_STATE = -16,        // call made in the wrong state (e.g. KV full)
  N730_COMM = -17,         // collective / peer error
};

// Precision ids of the .n730 format (per-tensor ids are the reference's).
enum : int {
  PREC_INT2 = 2, PREC_INT4 = 4, PREC_INT8 = 8, PREC_FP16 = 16,
  PREC_INT2_G = 0x42, PREC_INT4_G = 0x44, PREC_INT8_G = 0x48,
};

namespace n730 {

void set_error(const char* fmt, ...);
const char* last_error();

inline int cuda_rc(cudaError_t e, const char* what, int line) {
  if (e == cudaSuccess) return N730_OK;
  set_error("CUDA error at %s:%d: %s", what, line, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? N730_OOM : N730_CUDA_ERR;
}

#define N730_CUDA(x)                                            \
  do {                                                          \
    int _rc = ::n730::cuda_rc((x), __FILE__, __LINE__);         \
    if (_rc) return _rc;                                        \
  } while (0)

#define N730_CHECK_LAUNCH() N730_CUDA(cudaGetLastError())

#define N730_REQUIRE(cond, code, ...)                           \
  do {                                                          \
    if (!(cond)) { ::n730::set_error(__VA_ARGS__); return (code); } \
  } while (0)

inline int prec_bits(int prec) {
  switch (prec) {
    case PREC_INT2: case PREC_INT2_G: return 2;
    case PREC_INT4: case PREC_INT4_G: return 4;
    case PREC_INT8: case PREC_INT8_G: return 8;
    case PREC_FP16: return 16;
    default: return 0;
  }
}
inline bool prec_grouped(int prec) {
  return prec == PREC_INT2_G || prec == PREC_INT4_G || prec == PREC_INT8_G;
}

static inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Set kernel Kern's dynamic shared-memory limit to `bytes` once per device.
// The attribute belongs to the device that is current when it is set, so a
// process driving several GPUs sets it on each of them before its first launch
// there.  Thread-safe.
constexpr int N730_MAX_DEVICES = 128;
template <auto Kern>
int smem_attr_once(int bytes) {
  static std::mutex mu;
  static bool done[N730_MAX_DEVICES] = {};
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < N730_MAX_DEVICES, N730_BAD_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!done[dev]) {
    N730_CUDA(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev] = true;
  }
  return N730_OK;
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
// 16-byte streaming load that bypasses L1 (weights are read exactly once per step).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (a & mask) | orv
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}

// Exponent-field constant whose mantissa bit `pos` has weight 1:
// as_float((code << pos) | magic_bits(pos)) - magic_value(pos) == code exactly,
// valid while the code lies within mantissa bits [pos, 22].
__host__ __device__ constexpr uint32_t magic_bits(int pos) { return (uint32_t)(150 - pos) << 23; }
__host__ __device__ constexpr float magic_value_pow2(int e) {
  return e >= 0 ? (float)(1u << e) : 1.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// Programmatic dependent launch: wait for the producing grid / let the next start.
__device__ __forceinline__ void pdl_wait() {
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_launch_dependents() {
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
}

}  // namespace n730

namespace n730 {

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, 1-D) helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> shared, completion signalled on `bar` (tx bytes).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
               " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: false if the phase did not complete within `max_iter` polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_iter) {
  for (uint32_t i = 0; i < max_iter; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Device error word written by kernels whose bounded waits ran out.
enum : int { DEV_ERR_NONE = 0, DEV_ERR_TIMEOUT = 1 };

}  // namespace n730
