// One-shot allreduce over NVLink peer memory for tensor-parallel decode.
//
// The reference runs on one GPU and has no tensor parallelism.  Here the
// row-split projections (o_proj, down_proj) of a tensor-parallel decoder end
// with one sum of every rank's partial output.  For decode-sized messages
// (batch x hidden fp32, 32 KB at batch 1 for the 72B shape) an NCCL allreduce
// is latency-bound; here one kernel does the exchange and the residual add:
//
//   CTA s owns slice s of the vector.  It stores its slice of this rank's
//   partial into recv[par][rank] of EVERY rank (plain stores to peer memory
//   mapped with CUDA IPC), fences at system scope, and raises flags[par][rank][s]
//   = epoch on every rank.  It then waits, bounded, until flags[par][r][s] >=
//   epoch for all r in its own region, and adds the n partials of its slice in
//   rank order to x (deterministic, identical on every rank).
//
// Epochs count the ops done on this rank (device counter, updated by the op's
// last CTA, so graph replays see fresh epochs).  Slots alternate by epoch
// parity: a rank can be at most one op ahead of any other (it cannot finish op
// e+1 before every rank pushed op e+1, which each does only after finishing op
// e), so the slot a fast rank writes is never the one a slow rank still reads.
// No TMA, no multicast: plain loads and stores.
#include "common.cuh"
#include "tp_allreduce.h"

#include <vector>

namespace n730 {

constexpr uint64_t AR_WAIT_NS = 2000000000ull;  // a peer that never arrives: error after 2 s

__device__ __forceinline__ uint64_t ar_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ar_ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ar_st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.b32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256) ar_push_reduce_kernel(const ArArgs a) {
  __shared__ int s_ok;
  const int s = blockIdx.x, tid = threadIdx.x;
  const int epoch = *reinterpret_cast<volatile int*>(a.epoch) + 1, par = epoch & 1;
  // slice [lo, hi) in float4 units
  const int n4 = a.n >> 2;
  const int lo = (int)((int64_t)n4 * s / AR_SLICES), hi = (int)((int64_t)n4 * (s + 1) / AR_SLICES);
  const float4* src = reinterpret_cast<const float4*>(a.part);
  for (int r = 0; r < a.size; ++r) {
    float4* dst = reinterpret_cast<float4*>(a.peer[r].recv + ((int64_t)par * a.size + a.rank) * a.cap);
    for (int i = lo + tid; i < hi; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();  // this thread's pushes are visible to every rank before its flag
  __syncthreads();
  if (tid < a.size) ar_st_relaxed_sys(a.peer[tid].flags + ((int64_t)par * a.size + a.rank) * AR_SLICES + s, epoch);
  if (tid == 0) {  // every rank's slice s has arrived here
    bool ok = true;
    uint64_t t0 = 0;
    const uint64_t limit = a.wait_ns ? a.wait_ns : AR_WAIT_NS;
    for (int r = 0; r < a.size && ok; ++r) {
      const int* f = a.local.flags + ((int64_t)par * a.size + r) * AR_SLICES + s;
      while (ar_ld_relaxed_sys(f) < epoch) {
        const uint64_t t = ar_timer();
        if (!t0) t0 = t;
        else if (t - t0 > limit) { atomicExch(a.err, DEV_ERR_TIMEOUT); ok = false; break; }
      }
    }
    __threadfence_system();
    s_ok = ok;
  }
  __syncthreads();
  if (s_ok) {
    float4* x4 = reinterpret_cast<float4*>(a.x);
    for (int i = lo + tid; i < hi; i += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.size; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.local.recv + ((int64_t)par * a.size + r) * a.cap) + i);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      float4 h = x4[i];
      h.x += acc.x; h.y += acc.y; h.z += acc.z; h.w += acc.w;
      x4[i] = h;
    }
  }
  // the op's last CTA records the epoch for the next op (every CTA read it above)
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.done, 1) == AR_SLICES - 1) {
      *a.done = 0;
      *a.epoch = epoch;
      __threadfence();
    }
  }
}

static size_t ar_flag_words(int size) { return (size_t)2 * size * AR_SLICES; }
static size_t ar_head_bytes(int size) { return ((ar_flag_words(size) + 1) * sizeof(int) + 255) / 256 * 256; }

size_t ar_region_bytes(int size, int64_t cap) {
  return ar_head_bytes(size) + (size_t)2 * size * cap * sizeof(float);
}

ArRegion ar_region_at(void* base, int size) {
  ArRegion r;
  r.flags = reinterpret_cast<int*>(base);
  r.xcnt = r.flags + ar_flag_words(size);
  r.recv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base) + ar_head_bytes(size));
  return r;
}

int ar_launch(const ArArgs& a, cudaStream_t st) {
  N730_REQUIRE(a.size >= 2 && a.size <= AR_MAX_RANKS && a.n % 4 == 0 && a.n <= a.cap, N730_BAD_ARG,
               "tp allreduce: %d elements, %d ranks, capacity %lld", a.n, a.size, (long long)a.cap);
  ar_push_reduce_kernel<<<AR_SLICES, 256, 0, st>>>(a);
  N730_CUDA(cudaGetLastError());
  return N730_OK;
}

int* gemv_err_word();
int gemv_check_error(bool reset);

}  // namespace n730

using namespace n730;

// Self-check of the bounded peer wait (no counterpart in the reference): one
// 64-element op of the one-shot allreduce as rank 0 of 2, both regions local
// buffers of this process.  peer_arrives = 0: nothing ever writes "rank 1"'s
// flags, so every slice's wait runs out after wait_ns and the op returns
// N730_TIMEOUT through the device error word (the context stays usable);
// peer_arrives = 1: rank 1's flags and partial sums are written beforehand, so
// the op completes and x = part + peer part is checked (N730_BAD_ARG if not).
N730_API int n730_tp_wait_check(int64_t wait_ns, int peer_arrives, void* stream) {
  N730_REQUIRE(wait_ns > 0 && wait_ns <= 10000000000ll, N730_BAD_ARG, "tp_wait_check: wait %lld ns", (long long)wait_ns);
  cudaStream_t st = (cudaStream_t)stream;
  const int n = 64, size = 2;
  const size_t rb = ar_region_bytes(size, n);
  uint8_t* mem = nullptr;
  const size_t bytes = 2 * rb + 2 * n * sizeof(float) + 2 * sizeof(int);
  N730_CUDA(cudaMalloc(&mem, bytes));
  int rc = N730_OK;
  ArArgs a{};
  a.local = ar_region_at(mem, size);
  a.peer[0] = a.local;
  a.peer[1] = ar_region_at(mem + rb, size);
  float* part = reinterpret_cast<float*>(mem + 2 * rb);
  a.part = part;
  a.x = part + n;
  a.n = n;
  a.rank = 0;
  a.size = size;
  a.cap = n;
  a.epoch = reinterpret_cast<int*>(part + 2 * n);
  a.done = a.epoch + 1;
  a.err = gemv_err_word();
  a.wait_ns = (uint64_t)wait_ns;
  std::vector<float> h(2 * n);
  for (int i = 0; i < n; ++i) { h[i] = 1.0f; h[n + i] = 0.0f; }
  std::vector<int> flags(2 * size * AR_SLICES, 0);
  std::vector<float> peer_part(n, 2.0f);
  if (!a.err) rc = N730_OOM;
  if (!rc) rc = cuda_rc(cudaMemsetAsync(mem, 0, bytes, st), __FILE__, __LINE__);
  if (!rc) rc = cuda_rc(cudaMemcpyAsync(part, h.data(), 2 * n * sizeof(float), cudaMemcpyHostToDevice, st), __FILE__, __LINE__);
  if (!rc && peer_arrives) {  // rank 1 of epoch 1 (parity 1) has pushed its slice into rank 0's region
    for (int s = 0; s < AR_SLICES; ++s) flags[(1 * size + 1) * AR_SLICES + s] = 1;
    rc = cuda_rc(cudaMemcpyAsync(a.local.flags, flags.data(), flags.size() * sizeof(int), cudaMemcpyHostToDevice, st),
                 __FILE__, __LINE__);
    if (!rc) rc = cuda_rc(cudaMemcpyAsync(a.local.recv + (1 * size + 1) * n, peer_part.data(), n * sizeof(float),
                                          cudaMemcpyHostToDevice, st), __FILE__, __LINE__);
  }
  if (!rc) rc = ar_launch(a, st);
  if (!rc) rc = cuda_rc(cudaStreamSynchronize(st), __FILE__, __LINE__);
  if (!rc) rc = gemv_check_error(true);
  if (!rc) {
    rc = cuda_rc(cudaMemcpy(h.data(), part + n, n * sizeof(float), cudaMemcpyDeviceToHost), __FILE__, __LINE__);
    for (int i = 0; i < n && !rc; ++i)
      if (h[i] != 3.0f) { set_error("tp_wait_check: sum %g at %d, want 3", h[i], i); rc = N730_BAD_ARG; }
  }
  cudaStreamSynchronize(st);
  cudaFree(mem);
  return rc;
}
