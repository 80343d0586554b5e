// Next-token sampling on the GPU: greedy (argmax) or temperature + nucleus
// (top-p), the reference's host sampler (src-code/inference.py:674-682) run
// where the logits are, so a decode step returns token ids (4 bytes per
// sequence) instead of the whole logits row (608 KB at a 152k vocabulary).
//
// Semantics (per row, V logits l):
//   temp <= 0 : the first index of the largest logit (np.argmax).
//   else      : p_i = exp((l_i - max l) / temp); the tokens ordered by p
//               descending (ties by index); the nucleus is the shortest prefix
//               whose mass reaches top_p of the total (the reference's
//               searchsorted(cumsum, top_p) + 1); with u uniform in [0, 1),
//               the token is the first of the nucleus whose cumulative mass
//               exceeds u times the nucleus mass (numpy's choice rule:
//               searchsorted(cdf, u, 'right')).
// u comes from a counter-based hash of (seed, counter, row) and is written out
// when asked, so a checker can replay the choice.
//
// One CTA of 1024 threads per row, no full sort: masses are summed in 32.40
// fixed point (order-independent, deterministic) into 4096 bins of
// t = -64 (l - max) / temp (bin floor(t); the last bin also takes t >= 4095,
// masses below 2^-41 round to 0); a scan over the bins finds the bin where the
// cumulative mass crosses the cut (and later the sample point); only that
// bin's elements are gathered and bitonic-sorted in shared memory.  A bin with
// more than SP_CAP elements is split into 4096 finer bins once; elements that
// still fall together (equal to ~4e-6 relative) are taken in index order.
// Every pass reads the row from global memory (L2: the lm_head just wrote it).
#include <cmath>

#include "common.cuh"

namespace n730 {

constexpr int SP_THREADS = 1024;
constexpr int SP_BINS = 4096;
constexpr int SP_CAP = 4096;
constexpr double SP_ONE = 1099511627776.0;  // 2^40: fixed-point unit of probability mass

struct SpSmem {
  unsigned long long mass[SP_BINS];
  unsigned int cnt[SP_BINS];
  float key[SP_CAP];
  int idx[SP_CAP];
  unsigned long long wsum[32];
  float wmax[32];
  int widx[32];
  int n_gather;
  int first;
  unsigned long long res_cum;
  int res_idx;
};

__device__ __forceinline__ unsigned long long sp_mass(float p) {
  return (unsigned long long)((double)p * SP_ONE + 0.5);
}

// splitmix64 finaliser of (seed, counter, row): 24 random bits -> u in [0, 1)
__device__ __forceinline__ float sp_uniform(unsigned long long seed, unsigned long long counter, int row) {
  unsigned long long x = seed ^ (counter * 0x9E3779B97F4A7C15ull) ^ ((unsigned long long)row * 0xD1B54A32D192ED03ull);
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (float)(x >> 40) * (1.0f / 16777216.0f);
}

// Exclusive block scan of one u64 per thread; returns the exclusive prefix, *total the sum.
__device__ unsigned long long sp_scan(unsigned long long v, SpSmem& s, unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();
  if (lane == 31) s.wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = s.wsum[lane], wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    s.wsum[lane] = wi - w;  // exclusive prefix of the warp totals
    if (lane == 31) s.res_cum = wi;
  }
  __syncthreads();
  const unsigned long long ex = s.wsum[warp] + inc - v;
  *total = s.res_cum;
  __syncthreads();
  return ex;
}

// t = 64 (max - l) / temp, the bin coordinate (the same expression in every pass)
__device__ __forceinline__ float sp_t(float l, float m, float temp) {
  const float z = (l - m) / temp;
  return -z * 64.f;
}

// The elements selected by `pred(l, t)`, ordered by p descending and index
// ascending, gathered (n <= SP_CAP of them), sorted in shared memory and
// scanned: the first whose cumulative mass from `base` reaches `target`
// (strict: exceeds it) goes to s.res_idx, its inclusive cumulative mass to
// s.res_cum (rounding that leaves no crossing picks the last element).
template <class Pred>
__device__ void sp_sorted_pick(const float* row, int V, float m, float temp, Pred pred, unsigned long long base,
                               double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  if (tid == 0) s.n_gather = 0;
  __syncthreads();
  for (int i = tid; i < V; i += SP_THREADS) {
    const float l = row[i];
    if (pred(l, sp_t(l, m, temp))) {
      const int k = atomicAdd(&s.n_gather, 1);
      s.key[k] = expf((l - m) / temp);
      s.idx[k] = i;
    }
  }
  __syncthreads();
  const int n = s.n_gather;
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  for (int k = n + tid; k < np2; k += SP_THREADS) { s.key[k] = -1.f; s.idx[k] = 0x7fffffff; }
  __syncthreads();
  for (int sz = 2; sz <= np2; sz <<= 1) {
    for (int st = sz >> 1; st > 0; st >>= 1) {
      for (int k = tid; k < np2; k += SP_THREADS) {
        const int j = k ^ st;
        if (j > k) {
          const bool desc = (k & sz) == 0;  // this block's direction
          const float ka = s.key[k], kb = s.key[j];
          const int ia = s.idx[k], ib = s.idx[j];
          const bool a_first = ka > kb || (ka == kb && ia < ib);
          if (desc != a_first) { s.key[k] = kb; s.key[j] = ka; s.idx[k] = ib; s.idx[j] = ia; }
        }
      }
      __syncthreads();
    }
  }
  unsigned long long mm[4], loc = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int k = tid * 4 + r;
    mm[r] = k < n ? sp_mass(s.key[k]) : 0ull;
    loc += mm[r];
  }
  unsigned long long tot;
  const unsigned long long ex = sp_scan(loc, s, &tot);
  if (tid == 0) s.first = 0x7fffffff;
  __syncthreads();
  unsigned long long c = base + ex;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int k = tid * 4 + r;
    c += mm[r];
    if (k < n && (strict ? (double)c > target : (double)c >= target)) { atomicMin(&s.first, k); break; }
  }
  __syncthreads();
  const int k = s.first == 0x7fffffff ? max(n - 1, 0) : s.first;
  __syncthreads();
  if (tid == k / 4) {
    unsigned long long cc = base + ex;
    for (int r = 0; r <= k % 4; ++r) cc += mm[r];
    s.res_idx = n ? s.idx[k] : 0;
    s.res_cum = cc;
  }
  __syncthreads();
}

// The same pick over the elements of `pred` taken in index order (for values
// equal to within the finest bin, where the order by value is not resolved).
template <class Pred>
__device__ void sp_index_pick(const float* row, int V, float m, float temp, Pred pred, unsigned long long base,
                              double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  for (int c0 = 0; c0 < V; c0 += SP_THREADS) {
    const int i = c0 + tid;
    unsigned long long v = 0;
    if (i < V) {
      const float l = row[i];
      if (pred(l, sp_t(l, m, temp))) v = sp_mass(expf((l - m) / temp));
    }
    unsigned long long tot;
    const unsigned long long ex = sp_scan(v, s, &tot);
    if (tid == 0) s.first = 0x7fffffff;
    __syncthreads();
    const unsigned long long c = base + ex + v;
    if (v && (strict ? (double)c > target : (double)c >= target)) atomicMin(&s.first, i);
    __syncthreads();
    const int f = s.first;
    __syncthreads();
    if (f != 0x7fffffff) {
      if (i == f) { s.res_idx = f; s.res_cum = c; }
      __syncthreads();
      return;
    }
    base += tot;
  }
  if (tid == 0) { s.res_idx = V - 1; s.res_cum = base; }
  __syncthreads();
}

// Among the row's elements with t in [lo, hi) (hi < 0: no upper limit), ordered
// by p descending and index ascending, the first whose cumulative mass from
// `base` reaches `target` (strict: exceeds it): s.res_idx, s.res_cum.
__device__ void sp_find(const float* row, int V, float m, float temp, float lo, float hi, unsigned long long base,
                        double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  auto in_range = [lo, hi](float, float t) { return t >= lo && (hi < 0.f || t < hi); };
  if (tid == 0) s.n_gather = 0;
  __syncthreads();
  int cnt = 0;
  for (int i = tid; i < V; i += SP_THREADS) cnt += in_range(0.f, sp_t(row[i], m, temp));
  if (cnt) atomicAdd(&s.n_gather, cnt);
  __syncthreads();
  const int n = s.n_gather;
  __syncthreads();
  if (n <= SP_CAP) {
    sp_sorted_pick(row, V, m, temp, in_range, base, target, strict, s);
    return;
  }
  if (hi < 0.f) {  // the open last bin (masses ~0): index order
    sp_index_pick(row, V, m, temp, in_range, base, target, strict, s);
    return;
  }
  // too many elements: 4096 finer bins over [lo, hi), then the one holding the crossing
  const float w = (hi - lo) / (float)SP_BINS;
  auto sub = [lo, w](float t) { return min(SP_BINS - 1, max(0, (int)((t - lo) / w))); };
  for (int b = tid; b < SP_BINS; b += SP_THREADS) { s.mass[b] = 0ull; s.cnt[b] = 0u; }
  __syncthreads();
  for (int i = tid; i < V; i += SP_THREADS) {
    const float l = row[i];
    const float t = sp_t(l, m, temp);
    if (in_range(l, t)) {
      const int b = sub(t);
      atomicAdd(&s.mass[b], sp_mass(expf((l - m) / temp)));
      atomicAdd(&s.cnt[b], 1u);
    }
  }
  __syncthreads();
  unsigned long long mb[4], loc = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) { mb[r] = s.mass[tid * 4 + r]; loc += mb[r]; }
  unsigned long long tot;
  const unsigned long long ex = sp_scan(loc, s, &tot);
  if (tid == 0) s.first = 0x7fffffff;
  __syncthreads();
  unsigned long long c = base + ex;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    c += mb[r];
    if (strict ? (double)c > target : (double)c >= target) { atomicMin(&s.first, tid * 4 + r); break; }
  }
  __syncthreads();
  const int b = s.first == 0x7fffffff ? SP_BINS - 1 : s.first;
  __syncthreads();
  if (tid == b / 4) {
    unsigned long long cc = base + ex;
    for (int r = 0; r < b % 4; ++r) cc += mb[r];
    s.res_cum = cc;
  }
  __syncthreads();
  const unsigned long long before = s.res_cum;
  const unsigned int nb = s.cnt[b];
  __syncthreads();
  auto in_sub = [in_range, sub, b](float l, float t) { return in_range(l, t) && sub(t) == b; };
  if (nb <= (unsigned)SP_CAP) sp_sorted_pick(row, V, m, temp, in_sub, before, target, strict, s);
  else sp_index_pick(row, V, m, temp, in_sub, before, target, strict, s);
}

__global__ void __launch_bounds__(SP_THREADS, 1)
sample_kernel(const float* logits, int ld, int V, float temp, float top_p, unsigned long long seed,
              unsigned long long counter, int32_t* tokens, float* u_out) {
  extern __shared__ __align__(16) uint8_t sp_raw[];
  SpSmem& s = *reinterpret_cast<SpSmem*>(sp_raw);
  const int row_i = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = logits + (int64_t)row_i * ld;
  // 1. max and its first index
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += SP_THREADS) {
    const float v = row[i];
    if (v > bv) { bv = v; bi = i; }  // strided: the first index of this thread's maximum
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { s.wmax[warp] = bv; s.widx[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = s.wmax[lane];
    bi = s.widx[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s.wmax[0] = bv; s.widx[0] = bi; }
  }
  __syncthreads();
  const float m = s.wmax[0];
  const int amax = s.widx[0];
  const float u = temp > 0.f ? sp_uniform(seed, counter, row_i) : 0.f;
  if (tid == 0 && u_out) u_out[row_i] = u;
  if (!(temp > 0.f)) {
    if (tid == 0) tokens[row_i] = amax;
    return;
  }
  // 2. masses per bin
  for (int b = tid; b < SP_BINS; b += SP_THREADS) { s.mass[b] = 0ull; s.cnt[b] = 0u; }
  __syncthreads();
  for (int i = tid; i < V; i += SP_THREADS) {
    const float l = row[i];
    const float t = sp_t(l, m, temp);
    const int b = t < (float)(SP_BINS - 1) ? max(0, (int)t) : SP_BINS - 1;  // NaN: the last bin
    atomicAdd(&s.mass[b], sp_mass(expf((l - m) / temp)));
    atomicAdd(&s.cnt[b], 1u);
  }
  __syncthreads();
  unsigned long long mb[4], loc = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) { mb[r] = s.mass[tid * 4 + r]; loc += mb[r]; }
  unsigned long long total;
  const unsigned long long ex = sp_scan(loc, s, &total);
  // 3. nucleus: the bin where the cumulative mass reaches top_p of the total, then the element
  unsigned long long nucleus = total;
  if (top_p < 1.f) {
    const double target = (double)top_p * (double)total;
    if (tid == 0) s.first = 0x7fffffff;
    __syncthreads();
    unsigned long long c = ex;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      c += mb[r];
      if ((double)c >= target) { atomicMin(&s.first, tid * 4 + r); break; }
    }
    __syncthreads();
    const int b = s.first == 0x7fffffff ? SP_BINS - 1 : s.first;
    __syncthreads();
    if (tid == b / 4) {
      unsigned long long cc = ex;
      for (int r = 0; r < b % 4; ++r) cc += mb[r];
      s.res_cum = cc;
    }
    __syncthreads();
    const unsigned long long before = s.res_cum;
    __syncthreads();
    sp_find(row, V, m, temp, (float)b, b == SP_BINS - 1 ? -1.f : (float)(b + 1), before, target, false, s);
    nucleus = s.res_cum;
  }
  // 4. the sample: first element of the nucleus whose cumulative mass exceeds u * nucleus
  const double r = (double)u * (double)nucleus;
  if (tid == 0) s.first = 0x7fffffff;
  __syncthreads();
  {
    unsigned long long c = ex;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      c += mb[q];
      if ((double)c > r) { atomicMin(&s.first, tid * 4 + q); break; }
    }
  }
  __syncthreads();
  const int b = s.first == 0x7fffffff ? SP_BINS - 1 : s.first;
  __syncthreads();
  if (tid == b / 4) {
    unsigned long long cc = ex;
    for (int q = 0; q < b % 4; ++q) cc += mb[q];
    s.res_cum = cc;
  }
  __syncthreads();
  const unsigned long long before = s.res_cum;
  __syncthreads();
  sp_find(row, V, m, temp, (float)b, b == SP_BINS - 1 ? -1.f : (float)(b + 1), before, r, true, s);
  if (tid == 0) tokens[row_i] = s.res_idx;
}

int sample_launch(const float* d_logits, int batch, int vocab, int ld, float temp, float top_p,
                  unsigned long long seed, unsigned long long counter, int32_t* d_tokens, float* d_u,
                  cudaStream_t st) {
  N730_REQUIRE(d_logits && d_tokens, N730_NULL, "sample: null pointer");
  N730_REQUIRE(batch >= 1 && batch <= 65535 && vocab >= 1 && ld >= vocab, N730_BAD_ARG,
               "sample: batch %d, vocab %d, ld %d", batch, vocab, ld);
  N730_REQUIRE(std::isfinite(temp) && std::isfinite(top_p) && top_p > 0.f, N730_BAD_ARG,
               "sample: temperature %g, top_p %g", temp, top_p);
  if (int rc = smem_attr_once<sample_kernel>((int)sizeof(SpSmem))) return rc;
  sample_kernel<<<batch, SP_THREADS, sizeof(SpSmem), st>>>(d_logits, ld, vocab, temp, top_p, seed, counter, d_tokens,
                                                           d_u);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

}  // namespace n730

using namespace n730;

N730_API int n730_sample(const float* d_logits, int batch, int vocab, int ld, float temperature, float top_p,
                         uint64_t seed, uint64_t counter, int32_t* d_tokens, float* d_u, void* stream) {
  return sample_launch(d_logits, batch, vocab, ld, temperature, top_p, seed, counter, d_tokens, d_u,
                       (cudaStream_t)stream);
}
