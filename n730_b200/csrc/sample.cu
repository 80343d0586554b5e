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
// Three kernels per call, no full sort.  The two passes that touch every logit
// with arithmetic run on 64 CTAs per row (sp_stats_kernel: max / argmax / min
// of each slice; sp_hist_kernel: bin masses), the pick on one CTA of 1024
// threads per row (sample_kernel).  Masses are summed in 32.40
// fixed point (order-independent, deterministic) into 4096 bins of
// t = -64 (l - max) / temp spread over the row's own range (its smallest logit,
// capped where masses fall below 2^-43), so a near-flat row uses all bins; a
// scan over the bins finds the bin where the cumulative mass crosses the cut
// (and later the sample point); only that bin's elements are gathered and
// bitonic-sorted in shared memory.  A bin with more than SP_CAP elements is
// split into 4096 finer bins once; elements that still fall together (equal
// to a few 1e-7 relative) are taken in index order, as are rows of equal
// logits.  The pick reads the row two to four more times (L2: the lm_head just
// wrote it).  The
// temperature is applied as a multiplication by its reciprocal, so p can
// differ from exp((l - max) / temp) by an ulp or two.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace n730 {

constexpr int SP_THREADS = 1024;
constexpr int SP_BINS = 4096;
constexpr int SP_CAP = 4096;
constexpr float SP_ONE = 1099511627776.f;  // 2^40: fixed-point unit of probability mass
constexpr float SP_TMAX = 1920.f;          // bin range cap: t = 1920 is z = -30 (p < 2^-43)

struct SpSmem {
  unsigned long long mass[SP_BINS];
  float key[SP_CAP];
  int idx[SP_CAP];
  unsigned long long wsum[32];
  float wmax[32];
  float wmin[32];
  int widx[32];
  int n_gather;
  int first;
  int first_member;
  unsigned long long res_cum;
  int res_idx;
};

// p in [0, 1] in 32.40 fixed point: p * 2^40 is exact in fp32 (an exponent shift),
// so the conversion rounds the exact value
__device__ __forceinline__ unsigned long long sp_mass(float p) { return __float2ull_rn(p * SP_ONE); }

// splitmix64 finaliser of (seed, counter, row): 24 random bits -> u in [0, 1)
__device__ __forceinline__ float sp_uniform(unsigned long long seed, unsigned long long counter, int row) {
  unsigned long long x = seed ^ (counter * 0x9E3779B97F4A7C15ull) ^ ((unsigned long long)row * 0xD1B54A32D192ED03ull);
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (float)(x >> 40) * (1.0f / 16777216.0f);
}

// Row geometry: p(l) = exp((l - m) / temp) (by the reciprocal), and the bin
// coordinate x = (m - l) * sx: 4096 bins of width 1 over the row's spread
// [0, min(64 (m - min l) / temp, SP_TMAX)) scaled to [0, 4096); the last bin also
// takes everything beyond.  Sized to the row, so a near-flat row spreads over
// all bins instead of piling into a few.
struct SpGeom { float m, inv_temp, sx; };
__device__ __forceinline__ float sp_p(float l, const SpGeom& g) { return expf((l - g.m) * g.inv_temp); }
__device__ __forceinline__ float sp_x(float l, const SpGeom& g) { return (g.m - l) * g.sx; }
__device__ __forceinline__ int sp_bin_of(float x) {
  return x < (float)(SP_BINS - 1) ? max(0, (int)x) : SP_BINS - 1;  // NaN: the last bin
}
// finer bin inside bin b (from the same x as the bin, so the two never disagree)
__device__ __forceinline__ int sp_sub_of(float x, int b) {
  const float f = (x - (float)b) * (float)SP_BINS;
  return f < (float)(SP_BINS - 1) ? max(0, (int)f) : SP_BINS - 1;
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

// The elements selected by `pred(l)`, ordered by p descending and index
// ascending, gathered into shared memory (false, nothing picked, when there are
// more than SP_CAP of them), bitonic-sorted and scanned: the first whose
// cumulative mass from `base` reaches `target` (strict: exceeds it) goes to
// s.res_idx, its inclusive cumulative mass to s.res_cum (rounding that leaves
// no crossing picks the last element).
template <class Pred>
__device__ bool sp_sorted_pick(const float* row, int V, const SpGeom& g, Pred pred, unsigned long long base,
                               double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  if (tid == 0) s.n_gather = 0;
  __syncthreads();
  for (int i = tid; i < V; i += SP_THREADS) {
    const float l = row[i];
    if (pred(l)) {
      const int k = atomicAdd(&s.n_gather, 1);
      if (k < SP_CAP) { s.key[k] = sp_p(l, g); s.idx[k] = i; }
    }
  }
  __syncthreads();
  const int n = s.n_gather;
  if (n > SP_CAP) return false;
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
  return true;
}

// The same pick over the elements of `pred` taken in index order (values equal
// to within the finest bin, and rows of equal logits): thread t sums the members
// of its contiguous segment of the row, one block scan places the segments, and
// the thread whose segment holds the crossing walks it.
template <class Pred>
__device__ void sp_index_pick(const float* row, int V, const SpGeom& g, Pred pred, unsigned long long base,
                              double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  const int seg = (V + SP_THREADS - 1) / SP_THREADS;
  const int i0 = min(V, tid * seg), i1 = min(V, i0 + seg);
  auto cross = [strict, target](unsigned long long c) { return strict ? (double)c > target : (double)c >= target; };
  unsigned long long loc = 0;
  int first_member = 0x7fffffff;
  for (int i = i0; i < i1; ++i) {
    const float l = row[i];
    if (pred(l)) {
      loc += sp_mass(sp_p(l, g));
      first_member = min(first_member, i);
    }
  }
  unsigned long long tot;
  const unsigned long long ex = sp_scan(loc, s, &tot);
  if (tid == 0) { s.first = 0x7fffffff; s.first_member = 0x7fffffff; }
  __syncthreads();
  const unsigned long long c0 = base + ex, c1 = c0 + loc;
  if (!cross(c0) && cross(c1)) atomicMin(&s.first, tid);
  if (first_member != 0x7fffffff) atomicMin(&s.first_member, first_member);
  __syncthreads();
  if (s.first == 0x7fffffff) {  // crossed before the first member (its first member), or never (the last)
    if (tid == 0) {
      const bool before = cross(base);
      s.res_idx = before ? (s.first_member == 0x7fffffff ? 0 : s.first_member) : V - 1;
      s.res_cum = base + (before ? 0ull : tot);
    }
  } else if (tid == s.first) {
    unsigned long long c = c0;
    for (int i = i0; i < i1; ++i) {
      const float l = row[i];
      if (pred(l)) {
        c += sp_mass(sp_p(l, g));
        if (cross(c)) { s.res_idx = i; s.res_cum = c; break; }
      }
    }
  }
  __syncthreads();
}

// First bin (of masses mb[4] per thread, exclusive prefix ex) whose inclusive cumulative mass from
// `base` reaches `target` (strict: exceeds it); *before = the cumulative mass ahead of it.
__device__ int sp_cross_bin(const unsigned long long (&mb)[4], unsigned long long ex, unsigned long long base,
                            double target, bool strict, SpSmem& s, unsigned long long* before) {
  const int tid = threadIdx.x;
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
  *before = s.res_cum;
  __syncthreads();
  return b;
}

// Inside bin b (cumulative mass `base` ahead of it): the element where the
// cumulative mass reaches / exceeds `target` -> s.res_idx, s.res_cum.  A bin of
// more than SP_CAP elements is split into 4096 finer bins, and a finer bin that
// is still crowded is walked in index order.
__device__ void sp_pick_in_bin(const float* row, int V, const SpGeom& g, int b, unsigned long long base,
                               double target, bool strict, SpSmem& s) {
  const int tid = threadIdx.x;
  auto in_bin = [g, b](float l) { return sp_bin_of(sp_x(l, g)) == b; };
  if (sp_sorted_pick(row, V, g, in_bin, base, target, strict, s)) return;
  for (int q = tid; q < SP_BINS; q += SP_THREADS) s.mass[q] = 0ull;
  __syncthreads();
  for (int i = tid; i < V; i += SP_THREADS) {
    const float l = row[i];
    const float x = sp_x(l, g);
    if (sp_bin_of(x) == b) atomicAdd(&s.mass[sp_sub_of(x, b)], sp_mass(sp_p(l, g)));
  }
  __syncthreads();
  unsigned long long mb[4], loc = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) { mb[r] = s.mass[tid * 4 + r]; loc += mb[r]; }
  unsigned long long tot, before;
  const unsigned long long ex = sp_scan(loc, s, &tot);
  const int q = sp_cross_bin(mb, ex, base, target, strict, s, &before);
  auto in_sub = [g, b, q](float l) {
    const float x = sp_x(l, g);
    return sp_bin_of(x) == b && sp_sub_of(x, b) == q;
  };
  if (!sp_sorted_pick(row, V, g, in_sub, before, target, strict, s))
    sp_index_pick(row, V, g, in_sub, before, target, strict, s);  // values equal to a few 1e-7
}

// ---- row statistics and bin masses on many CTAs per row ----
// The finishing kernel below runs on one CTA per row; the two passes that touch
// every logit with real arithmetic (the max / argmax / min scan and the bin
// masses, one exp per logit) are spread over SP_SLICES CTAs per row first.
constexpr int SP_SLICES = 64;
constexpr int SP_PRE_THREADS = 256;

struct SpStat { float mx; int idx; float mn; int pad; };

// Fixed-order combination of a row's slice statistics: the largest logit with
// its first index (slices are consecutive index ranges), and the smallest.
__device__ __forceinline__ SpStat sp_combine(const SpStat* st) {
  SpStat r{-INFINITY, 0x7fffffff, INFINITY, 0};
  for (int k = 0; k < SP_SLICES; ++k) {
    const SpStat a = st[k];
    if (a.mx > r.mx || (a.mx == r.mx && a.idx < r.idx)) { r.mx = a.mx; r.idx = a.idx; }
    r.mn = fminf(r.mn, a.mn);
  }
  return r;
}

__device__ __forceinline__ void sp_slice(int V, int sl, int* i0, int* i1) {
  const int per = (V + SP_SLICES - 1) / SP_SLICES;
  *i0 = min(V, sl * per);
  *i1 = min(V, *i0 + per);
}

// grid (SP_SLICES, rows): slice statistics; also zeroes the slice's share of the
// row's bins for the next kernel
__global__ void __launch_bounds__(SP_PRE_THREADS)
sp_stats_kernel(const float* logits, int ld, int V, SpStat* stats, unsigned long long* hist) {
  __shared__ float wmx[SP_PRE_THREADS / 32], wmn[SP_PRE_THREADS / 32];
  __shared__ int widx[SP_PRE_THREADS / 32];
  const int sl = blockIdx.x, row_i = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = logits + (int64_t)row_i * ld;
  int i0, i1;
  sp_slice(V, sl, &i0, &i1);
  float bv = -INFINITY, mn = INFINITY;
  int bi = 0x7fffffff;
  for (int i = i0 + tid; i < i1; i += SP_PRE_THREADS) {
    const float v = row[i];
    if (v > bv) { bv = v; bi = i; }  // strided: the first index of this thread's maximum
    mn = fminf(mn, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  if (lane == 0) { wmx[warp] = bv; widx[warp] = bi; wmn[warp] = mn; }
  __syncthreads();
  if (tid == 0) {
    SpStat r{-INFINITY, 0x7fffffff, INFINITY, 0};
    for (int w = 0; w < SP_PRE_THREADS / 32; ++w) {
      if (wmx[w] > r.mx || (wmx[w] == r.mx && widx[w] < r.idx)) { r.mx = wmx[w]; r.idx = widx[w]; }
      r.mn = fminf(r.mn, wmn[w]);
    }
    stats[(size_t)row_i * SP_SLICES + sl] = r;
  }
  unsigned long long* h = hist + (size_t)row_i * SP_BINS;
  for (int b = sl * (SP_BINS / SP_SLICES) + tid; b < (sl + 1) * (SP_BINS / SP_SLICES); b += SP_PRE_THREADS) h[b] = 0ull;
}

// Row geometry from the combined statistics (the same arithmetic in every kernel,
// so every CTA of a row bins identically); false: greedy or a row of equal logits.
__device__ __forceinline__ bool sp_geom(const SpStat& t, float temp, SpGeom* g) {
  if (!(temp > 0.f)) return false;
  const float inv_temp = 1.0f / temp;
  const float R = fminf((t.mx - t.mn) * 64.f * inv_temp, SP_TMAX);
  if (!(R > 0.f)) return false;
  *g = SpGeom{t.mx, inv_temp, 64.f * inv_temp * ((float)SP_BINS / R)};
  return true;
}

// grid (SP_SLICES, rows): the slice's bin masses (32.40 fixed point) summed in
// shared memory, then added into the row's bins (integer sums: order-independent)
__global__ void __launch_bounds__(SP_PRE_THREADS)
sp_hist_kernel(const float* logits, int ld, int V, float temp, const SpStat* stats, unsigned long long* hist) {
  __shared__ unsigned long long hs[SP_BINS];
  __shared__ SpStat tot;
  const int sl = blockIdx.x, row_i = blockIdx.y, tid = threadIdx.x;
  const float* row = logits + (int64_t)row_i * ld;
  if (tid == 0) tot = sp_combine(stats + (size_t)row_i * SP_SLICES);
  for (int b = tid; b < SP_BINS; b += SP_PRE_THREADS) hs[b] = 0ull;
  __syncthreads();
  SpGeom g;
  if (!sp_geom(tot, temp, &g)) return;
  int i0, i1;
  sp_slice(V, sl, &i0, &i1);
  for (int i = i0 + tid; i < i1; i += SP_PRE_THREADS) {
    const float l = row[i];
    atomicAdd(&hs[sp_bin_of(sp_x(l, g))], sp_mass(sp_p(l, g)));
  }
  __syncthreads();
  unsigned long long* h = hist + (size_t)row_i * SP_BINS;
  for (int b = tid; b < SP_BINS; b += SP_PRE_THREADS)
    if (hs[b]) atomicAdd(h + b, hs[b]);
}

__global__ void __launch_bounds__(SP_THREADS, 1)
sample_kernel(const float* logits, int ld, int V, float temp, float top_p, unsigned long long seed,
              unsigned long long counter, int32_t* tokens, float* u_out, const SpStat* stats,
              const unsigned long long* hist) {
  extern __shared__ __align__(16) uint8_t sp_raw[];
  SpSmem& s = *reinterpret_cast<SpSmem*>(sp_raw);
  const int row_i = blockIdx.x, tid = threadIdx.x;
  const float* row = logits + (int64_t)row_i * ld;
  // 1. the largest logit with its first index, and the smallest (from the slice statistics)
  if (tid == 0) {
    const SpStat t = sp_combine(stats + (size_t)row_i * SP_SLICES);
    s.wmax[0] = t.mx;
    s.widx[0] = t.idx;
    s.wmin[0] = t.mn;
  }
  __syncthreads();
  const float m = s.wmax[0];
  const int amax = s.widx[0];
  const float lmin = s.wmin[0];
  __syncthreads();
  const float u = temp > 0.f ? sp_uniform(seed, counter, row_i) : 0.f;
  if (tid == 0 && u_out) u_out[row_i] = u;
  if (!(temp > 0.f)) {
    if (tid == 0) tokens[row_i] = amax;
    return;
  }
  const float inv_temp = 1.0f / temp;
  const float R = fminf((m - lmin) * 64.f * inv_temp, SP_TMAX);
  if (!(R > 0.f)) {
    // every logit equal: equal probabilities, taken in index order
    const SpGeom g{m, inv_temp, 0.f};
    auto all = [](float) { return true; };
    const unsigned long long total = (unsigned long long)V * sp_mass(1.f);
    unsigned long long nucleus = total;
    if (top_p < 1.f) {
      sp_index_pick(row, V, g, all, 0ull, (double)top_p * (double)total, false, s);
      nucleus = s.res_cum;
    }
    sp_index_pick(row, V, g, all, 0ull, (double)u * (double)nucleus, true, s);
    if (tid == 0) tokens[row_i] = s.res_idx;
    return;
  }
  const SpGeom g{m, inv_temp, 64.f * inv_temp * ((float)SP_BINS / R)};
  // 2. masses per bin (summed by sp_hist_kernel)
  unsigned long long mb[4], loc = 0;
  const unsigned long long* hrow = hist + (size_t)row_i * SP_BINS;
#pragma unroll
  for (int r = 0; r < 4; ++r) { mb[r] = hrow[tid * 4 + r]; loc += mb[r]; }
  unsigned long long total;
  const unsigned long long ex = sp_scan(loc, s, &total);
  // (mb / ex stay in registers: the finer bins of a crowded bin reuse s.mass)
  // 3. nucleus: where the cumulative mass reaches top_p of the total
  unsigned long long nucleus = total;
  if (top_p < 1.f) {
    const double target = (double)top_p * (double)total;
    unsigned long long before;
    const int b = sp_cross_bin(mb, ex, 0ull, target, false, s, &before);
    sp_pick_in_bin(row, V, g, b, before, target, false, s);
    nucleus = s.res_cum;
  }
  // 4. the sample: the first element whose cumulative mass exceeds u * nucleus
  const double r = (double)u * (double)nucleus;
  unsigned long long before;
  const int c = sp_cross_bin(mb, ex, 0ull, r, true, s, &before);
  sp_pick_in_bin(row, V, g, c, before, r, true, s);
  if (tid == 0) tokens[row_i] = s.res_idx;
}

// Per-device workspace of the pre-passes (slice statistics + row bins), grown on
// demand, never inside a stream capture.
static int sp_workspace(int batch, cudaStream_t st, SpStat** stats, unsigned long long** hist) {
  static std::mutex mu;
  static uint8_t* buf[N730_MAX_DEVICES] = {};
  static int cap[N730_MAX_DEVICES] = {};
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < N730_MAX_DEVICES, N730_BAD_ARG, "sample: device %d", dev);
  const size_t hist_off = ((size_t)batch * SP_SLICES * sizeof(SpStat) + 255) / 256 * 256;
  std::lock_guard<std::mutex> lk(mu);
  if (cap[dev] < batch) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    N730_CUDA(cudaStreamIsCapturing(st, &cs));
    N730_REQUIRE(cs == cudaStreamCaptureStatusNone, N730_STATE,
                 "sample: workspace for %d rows must grow outside stream capture", batch);
    N730_CUDA(cudaStreamSynchronize(st));  // a kernel in flight may still use the old buffer
    if (buf[dev]) N730_CUDA(cudaFree(buf[dev]));
    buf[dev] = nullptr;
    cap[dev] = 0;
    N730_CUDA(cudaMalloc(&buf[dev], hist_off + (size_t)batch * SP_BINS * 8));
    cap[dev] = batch;
  }
  const size_t off = ((size_t)cap[dev] * SP_SLICES * sizeof(SpStat) + 255) / 256 * 256;
  *stats = reinterpret_cast<SpStat*>(buf[dev]);
  *hist = reinterpret_cast<unsigned long long*>(buf[dev] + off);
  return N730_OK;
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
  SpStat* stats = nullptr;
  unsigned long long* hist = nullptr;
  if (int rc = sp_workspace(batch, st, &stats, &hist)) return rc;
  sp_stats_kernel<<<dim3(SP_SLICES, batch), SP_PRE_THREADS, 0, st>>>(d_logits, ld, vocab, stats, hist);
  N730_CHECK_LAUNCH();
  if (temp > 0.f) {
    sp_hist_kernel<<<dim3(SP_SLICES, batch), SP_PRE_THREADS, 0, st>>>(d_logits, ld, vocab, temp, stats, hist);
    N730_CHECK_LAUNCH();
  }
  sample_kernel<<<batch, SP_THREADS, sizeof(SpSmem), st>>>(d_logits, ld, vocab, temp, top_p, seed, counter, d_tokens,
                                                           d_u, stats, hist);
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
