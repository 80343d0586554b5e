// Persistent decode step: the whole batch-1 forward pass (every layer's qkv
// GEMV, RoPE + GQA attention, o_proj, gate|up + SwiGLU, down_proj, then the
// final-norm lm_head) in ONE cooperative launch of one 16-warp CTA per SM.
//
// Why: a decode step is ~140 dependent GEMVs that each stream a few MB of
// packed weights.  As separate kernels every op pays a launch, a prologue that
// re-reads x behind its own weight prefetch, and a pipeline fill.  Here:
//  * Each CTA owns a fixed run of whole row tiles of every GEMV, split evenly
//    over its 16 warps by [tile][group] units; lane 0 of each warp streams the
//    warp's chunks through a private TMA bulk-copy ring whose cursor runs
//    ACROSS ops and layers.  Weights never depend on activations, so while the
//    CTA waits at an op boundary its ring already holds the next op's weights.
//  * Ops are separated by a grid barrier (one arrival counter, bounded spin on
//    %globaltimer; an expired wait raises the abort flag that releases every
//    CTA and sets the device error word).  Each op then costs few dependent
//    global round trips: the barrier, one batch of loads (x, norm weights,
//    residual and bias rows), and fire-and-forget stores.
//  * After the barrier each CTA builds the op's fp16 x fragments and per-group
//    x sums (RMSNorm folded in) in shared memory; warps run the tensor-core
//    INT4 GEMV of mma_gemv.cuh on their chunks; a tile split between warps is
//    merged by the last contributor in warp order (deterministic) and written
//    with its epilogue (store, residual add in place, or SwiGLU of interleaved
//    gate/up rows).
//  * Attention: each split is one KV page (64 positions) of one KV head.  The
//    page's K and V are bulk-copied into shared memory a whole layer ahead (the
//    cached positions do not depend on this step); the split holding the new
//    position RoPEs and appends k/v; scores and P V on the tensor cores with an
//    online softmax; once every split of a head has published, each split
//    merges a slice of the head's outputs with one batch of loads:
//    out = sum_s e^(m_s-M) o_s / (sum_s e^(m_s-M) l_s + 1e-9)
//    (the reference normalisation, n730_cuda.cu:236-257).
//  * Template variant EXT = true adds what only some models need, so that the
//    INT4 single-GPU kernel carries none of it: phase tables read from global
//    memory (too large for shared memory), INT8 / FP16 weight tiles
//    (decode_persist.h), and the tensor-parallel exchange (a push epilogue into
//    every rank's exchange slot over peer memory, cross-GPU barriers on
//    counters in every rank's region, rank-order sums in the next prologue).
// Data written by other CTAs during the launch is read with ld.global.cg (L2),
// never through a possibly stale L1 line.
#include <algorithm>
#include <cmath>

#include "decode_persist.h"
#include "mma_gemv.cuh"
#include "qweight.h"

namespace n730 {

constexpr int PD_WARPS = 16;
constexpr int PD_THREADS = PD_WARPS * 32;
constexpr int PD_RING = 2;         // chunks in flight per warp
constexpr int PD_NREG = 4;         // normalised x items (4 values) per thread: K <= 4 * 512 * 4
constexpr int PD_KNORM = 4 * PD_THREADS * PD_NREG;
constexpr int PD_MAXG = 8;         // query heads per KV head
constexpr int PD_MAXSPLIT = 64;    // context splits per KV head
constexpr int PD_ADDMAX = 512;     // epilogue addend rows (bias / residual) per CTA
constexpr uint64_t PD_WAIT_NS = 200000000ull;  // grid-barrier wait limit (0.2 s)
// Thread roles outside the weight ring (each warp's lane 0 issues that warp's
// ring copies): the KV page copies are issued and waited for by PD_KV_T, and the
// grid-barrier arrival, split publication and exit handshake (the release
// fences) by PD_SYNC_T, a thread with no bulk copies of its own in flight.
constexpr int PD_KV_T = 1;
constexpr int PD_SYNC_T = 2;
constexpr float PD_FIX = 4294967296.0f;          // 32.32 fixed point of the FFN accumulator
constexpr float PD_UNFIX = 2.3283064365386963e-10f;

// groups per chunk: ~4.2-4.6 KB per bulk copy
__host__ __device__ constexpr int pd_gpc(int kpg) { return kpg == 4 ? 8 : kpg == 8 ? 4 : 2; }

// [lo, hi) split into n near-equal parts: start of part i.  32-bit unsigned
// arithmetic (the planner bounds (hi - lo) * n below 2^31).
__device__ __forceinline__ int pd_rng(int lo, int hi, int i, int n) {
  return lo + (int)((unsigned)(hi - lo) * (unsigned)i / (unsigned)n);
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *cnt >= target or the abort flag is raised: each poll issues the
// two relaxed loads together (one L2 round trip); once the count is reached one
// acquire load of it synchronises with the arrivals' release operations (an
// acq_rel fence would also wait for this thread's own arrival to complete).
// Raises the abort flag and the device error word after PD_WAIT_NS.
__device__ __forceinline__ bool pd_wait_count(const PdArgs& a, const int* cnt, int target) {
  uint64_t t0 = 0;
  bool ok = true;
  for (;;) {
    const int c = ld_relaxed(cnt), ab = ld_relaxed(&a.sync[2]);
    if (c >= target) break;
    if (ab) { ok = false; break; }
    const uint64_t t = gtimer();
    if (!t0) t0 = t;
    else if (t - t0 > PD_WAIT_NS) {
      atomicExch(&a.sync[2], 1);
      atomicExch(a.err, DEV_ERR_TIMEOUT);
      ok = false;
      break;
    }
  }
  if (ok) (void)ld_acquire(cnt);
  else asm volatile("fence.acq_rel.gpu;" ::: "memory");
  return ok;
}

// Grid barrier number k (all CTAs call it in the same order).  False when the
// launch is being aborted.
__device__ bool pd_barrier(const PdArgs& a, int k, int* flag, unsigned long long* t_arrive) {
  __syncthreads();
  if (threadIdx.x == PD_SYNC_T) {
    if (t_arrive) *t_arrive = gtimer();
    asm volatile("red.release.gpu.global.add.s32 [%0], 1;" :: "l"(&a.sync[0]) : "memory");
    *flag = pd_wait_count(a, &a.sync[0], (int)gridDim.x * k);
  }
  __syncthreads();
  return *flag != 0;
}

// Cross-GPU barrier number k of this launch (tensor parallel): every CTA of
// every rank arrives on every rank's counter (system-scope release after the
// CTA's peer stores), then waits until its own rank's counter shows all
// tp_size x grid arrivals.  The counters are never reset: launch e's barrier k
// completes at tp_size * grid * (e * n_xbar + k) (32-bit wrapping compare), so
// a rank that starts the next launch early cannot disturb a slow one.  Waits
// end after PD_XWAIT_NS (a peer whose launch never comes) with the abort flag
// and the device error word raised.  The limit covers the skew between the
// ranks' launches (host work between steps, graph instantiation: milliseconds)
// plus a whole step (72B at one rank: ~11 ms), with a wide margin.
constexpr uint64_t PD_XWAIT_NS = 2000000000ull;
__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ bool pd_xbarrier(const PdArgs& a, int xep, int k, int* flag, unsigned long long* t_arrive) {
  __syncthreads();
  if (threadIdx.x == PD_SYNC_T) {
    if (t_arrive) *t_arrive = gtimer();
    // one system-scope fence orders this CTA's pushes (ordered before it by the CTA barrier)
    // before all of its arrivals, which are then relaxed
    asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
    for (int r = 0; r < PD_MAX_RANKS; ++r)
      if (r < a.tp_size) asm volatile("red.relaxed.sys.global.add.s32 [%0], 1;" :: "l"(a.xcnt[r]) : "memory");
    const unsigned target = (unsigned)a.tp_size * gridDim.x * ((unsigned)xep * (unsigned)a.n_xbar + (unsigned)k);
    const int* cnt = a.xcnt_local;
    uint64_t t0 = 0;
    bool ok = true;
    for (;;) {
      const int c = ld_relaxed_sys(cnt), ab = ld_relaxed(&a.sync[2]);
      if ((int)((unsigned)c - target) >= 0) break;
      if (ab) { ok = false; break; }
      const uint64_t t = gtimer();
      if (!t0) t0 = t;
      else if (t - t0 > PD_XWAIT_NS) {
        atomicExch(&a.sync[2], 1);
        atomicExch(a.err, DEV_ERR_TIMEOUT);
        ok = false;
        break;
      }
    }
    // a completed wait ends with one acquire load of the counter, which synchronises with every
    // rank's release pattern (system fence, then relaxed arrivals); an aborted one with a fence
    if (ok) (void)ld_acquire_sys(cnt);
    else asm volatile("fence.acq_rel.sys;" ::: "memory");
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// This CTA's row tiles [t0, t1) of weight-streaming phase P: an even share of
// a GEMV's tiles, or for an FFN phase the gate|up tiles of the CTA's FFN
// groups (2 kpg tiles of 8 interleaved gate/up channel pairs per group).
__device__ __forceinline__ void pd_tiles(const PdPhase& P, int cta, int NC, int kpg, int& t0, int& t1) {
  if (P.kind == PD_FFN) {
    t0 = pd_rng(0, P.G2, cta, NC) * 2 * kpg;
    t1 = pd_rng(0, P.G2, cta + 1, NC) * 2 * kpg;
  } else {
    const int T = (P.rows + 15) >> 4;
    t0 = pd_rng(0, T, cta, NC);
    t1 = pd_rng(0, T, cta + 1, NC);
  }
}

// KV split geometry of this step (batch 1): ns splits per KV head of ppi pages.
struct PdSplits { int pos, L, npages, ppi, ns, items; };
__device__ __forceinline__ PdSplits pd_splits(const PdArgs& a) {
  PdSplits s;
  s.pos = a.seq_lens[0];
  s.L = s.pos + 1;
  s.npages = (s.L + PD_PAGE - 1) / PD_PAGE;
  const int ns0 = min(s.npages, a.max_split);
  s.ppi = (s.npages + ns0 - 1) / ns0;
  s.ns = (s.npages + s.ppi - 1) / s.ppi;
  s.items = a.d.n_kv * s.ns;
  return s;
}

// One INT8 unit (16 rows x KPG k-steps, PdTile layout) against x fragments xb
// (k-step pairs as in mma_chunk) and the x sum xs of its 128 columns:
// codes become fp16 1024 + q by a byte permute, so with C = sum (1024 + q) x,
// row r gets scale_r * (C - (1024 + zero_r) * xs).
template <int KPG>
__device__ __forceinline__ void pd_unit_i8(const uint8_t* u, int lane, const uint4* xb, float xs, float& y_g,
                                           float& y_g8) {
  constexpr uint32_t M = 0x64646464u;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s2 = 0; s2 < KPG / 2; ++s2) {
    const uint4 w = *reinterpret_cast<const uint4*>(u + (s2 * 32 + lane) * 16);
    const uint4 v = xb[s2 * 4];
    mma16816(c, __byte_perm(w.x, M, 0x5140), __byte_perm(w.x, M, 0x5342), __byte_perm(w.y, M, 0x5140),
             __byte_perm(w.y, M, 0x5342), v.x, v.y);
    mma16816(c, __byte_perm(w.z, M, 0x5140), __byte_perm(w.z, M, 0x5342), __byte_perm(w.w, M, 0x5140),
             __byte_perm(w.w, M, 0x5342), v.z, v.w);
  }
  const float4 sz = reinterpret_cast<const float4*>(u + 16 * PD_TILE_K)[lane >> 2];
  y_g = fmaf(sz.x, c[0] - (1024.f + sz.y) * xs, y_g);
  y_g8 = fmaf(sz.z, c[2] - (1024.f + sz.w) * xs, y_g8);
}

// One FP16 unit: the tiles are the A fragments themselves.
template <int KPG>
__device__ __forceinline__ void pd_unit_f16(const uint8_t* u, int lane, const uint4* xb, float& y_g, float& y_g8) {
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < KPG; ++s) {
    const uint4 w = *reinterpret_cast<const uint4*>(u + (s * 32 + lane) * 16);
    const uint4 v = xb[(s >> 1) * 4];
    mma16816(c, w.x, w.y, w.z, w.w, (s & 1) ? v.z : v.x, (s & 1) ? v.w : v.y);
  }
  y_g += c[0];
  y_g8 += c[2];
}

// EXT: the tensor-parallel exchange (push epilogue, cross-GPU barriers, rank
// sums), phase tables in global memory and INT8 / FP16 weight tiles; without
// it that code is compiled out.
template <int KPG, int HD, bool EXT>
__global__ void __launch_bounds__(PD_THREADS, 1) persist_decode_kernel(const PdArgs a) {
  constexpr int GPC = pd_gpc(KPG);
  constexpr int GB = KPG * 128 + 64;  // bytes per group
  constexpr int H2 = HD / 2;
  constexpr uint32_t PAGE_BYTES = PD_PAGE * HD * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NC = gridDim.x, cta = blockIdx.x;
  const int g = lane >> 2, tq = lane & 3;
  uint64_t* wb = reinterpret_cast<uint64_t*>(smem) + warp * PD_RING;
  uint64_t* kvbar = reinterpret_cast<uint64_t*>(smem) + PD_WARPS * PD_RING;
  uint8_t* ring = smem + a.ring_off + (size_t)warp * PD_RING * a.ring_stride;
  uint8_t* work = smem + a.work_off;
  __half* Ks = reinterpret_cast<__half*>(smem + a.kv_off);      // [PD_PAGE][HD]
  __half* Vs = Ks + PD_PAGE * HD;                               // [PD_PAGE][HD]
  float* addv = reinterpret_cast<float*>(smem + a.add_off);      // [PD_ADDMAX]
  float* wpart = reinterpret_cast<float*>(smem + a.wpart_off);  // [16 warps][2][16 rows]
  int* wcnt = reinterpret_cast<int*>(smem + a.misc_off);         // [16]
  int* flag = wcnt + 16;                                         // [16]
  float* red = reinterpret_cast<float*>(wcnt + 32);              // [32]
  int* wr = wcnt + 64;                                           // [PD_WARPS + 1] unit ranges of a GEMV phase
  // tracing: ns the warps spent waiting for weight chunks in this phase ([0] GEMV / gate|up, [1] down)
  unsigned long long* wacc = reinterpret_cast<unsigned long long*>(wcnt + 82);
  float* mloc = reinterpret_cast<float*>(smem + a.ffn_off);      // FFN: this CTA's SwiGLU channels

  const PdSplits sp = pd_splits(a);
  const AttnDims& d = a.d;
  const int GQ = d.n_heads / d.n_kv;
  const bool has_item = cta < sp.items;
  const int kvh = has_item ? cta / sp.ns : 0, split = has_item ? cta % sp.ns : 0;
  const int pg0 = split * sp.ppi, pg1 = min(sp.npages, pg0 + sp.ppi);

  // the phase table lives in shared memory: phase transitions read it on the
  // critical path (producer cursor and every phase's prologue)
  // (tables too large for shared memory are read from global memory)
  PdPhase* phs = !EXT || a.tab_off >= 0 ? reinterpret_cast<PdPhase*>(smem + a.tab_off)
                                        : const_cast<PdPhase*>(a.phases);
  if (!EXT || a.tab_off >= 0) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.phases);
    uint32_t* dst = reinterpret_cast<uint32_t*>(phs);
    const int words = a.n_phases * (int)(sizeof(PdPhase) / 4);
    for (int i = tid; i < words; i += PD_THREADS) dst[i] = __ldg(src + i);
  }
  if (tid < 16) wcnt[tid] = 0;
  if (lane == 0) {
    for (int r = 0; r < PD_RING; ++r) mbar_init(&wb[r], 1);
    if (warp == 0) mbar_init(kvbar, 1);
    fence_mbar_init();
  }
  if (a.trace && tid == PD_SYNC_T) a.trace[cta] = gtimer();  // launch start (phase 0 has no barrier)
  __syncthreads();

  // ---- KV page copies (PD_KV_T): page p of this CTA's KV head, layer of phase ph ----
  int kv_uses = 0;      // copies issued (PD_KV_T)
  int kv_waited = 0;    // copies waited for (PD_KV_T)
  auto kv_issue = [&](int ph, int p) {
    const PdPhase& P = phs[ph];
    const int page = a.block_table[p];
    const int64_t off = ((int64_t)page * d.n_kv + kvh) * PD_PAGE * HD;
    mbar_arrive_expect_tx(kvbar, 2 * PAGE_BYTES);
    bulk_g2s(Ks, P.kv.k_pages + off, PAGE_BYTES, kvbar);
    bulk_g2s(Vs, P.kv.v_pages + off, PAGE_BYTES, kvbar);
    ++kv_uses;
  };
  auto next_attn = [&](int ph) {
    for (; ph < a.n_phases; ++ph)
      if (phs[ph].kind == PD_ATTN) return ph;
    return a.n_phases;
  };

  // ---- weight stream: this warp's chunks of every GEMV / FFN op, in op order ----
  // sub 0: [tile][group] units of the phase's (gate|up) GEMV; sub 1: an FFN
  // phase's down_proj units, whole row tiles [u, end) of the warp, each the
  // CTA's nj groups from j0 (one bulk copy per tile).
  struct Cursor { int ph, sub, u, end, gi, G, j0, nj, gb, gpc; const uint8_t* blob; };
  // bytes and units per ring chunk of a phase's tiles (INT8 / FP16 tiles: EXT only)
  auto unit_bytes = [&](const PdPhase& P) {
    return !EXT || P.prec == 4 || P.prec == 0 ? GB : P.prec == 8 ? PD_UNIT8 : PD_UNIT16;
  };
  auto set_down = [&](Cursor& c, int ph) {
    const PdPhase& P = phs[ph];
    const int j0 = pd_rng(0, P.G2, cta, NC), j1 = pd_rng(0, P.G2, cta + 1, NC);
    const int Td = (P.rows2 + 15) >> 4;
    const int w0 = pd_rng(0, Td, warp, PD_WARPS), w1 = pd_rng(0, Td, warp + 1, PD_WARPS);
    if (j0 == j1 || w0 == w1) return false;
    // c.G: row tiles of down_proj, the stride of its group-major units
    c.ph = ph; c.sub = 1; c.u = w0; c.end = w1; c.gi = 0; c.G = Td; c.j0 = j0; c.nj = j1 - j0; c.blob = P.blob2;
    return true;
  };
  auto set_phase = [&](Cursor& c, int ph) {
    for (; ph < a.n_phases; ++ph) {
      const PdPhase& P = phs[ph];
      if (P.kind != PD_GEMV && P.kind != PD_FFN) continue;
      int t0, t1;
      pd_tiles(P, cta, NC, KPG, t0, t1);
      const int c0 = t0 * P.G, c1 = t1 * P.G;
      const int w0 = pd_rng(c0, c1, warp, PD_WARPS), w1 = pd_rng(c0, c1, warp + 1, PD_WARPS);
      if (w0 < w1) {
        c.ph = ph; c.sub = 0; c.u = w0; c.end = w1; c.gi = w0 % P.G; c.G = P.G; c.j0 = 0; c.nj = 0; c.blob = P.blob;
        c.gb = unit_bytes(P);
        c.gpc = EXT ? a.ring_stride / c.gb : GPC;
        return;
      }
      if (P.kind == PD_FFN && set_down(c, ph)) return;
    }
    c.ph = a.n_phases;
  };
  int issued = 0, consumed = 0;
  Cursor prod{0, 0, 0, 0, 0, 1, 0, 0, GB, GPC, nullptr};
  auto issue_next = [&](int slot) {  // lane 0
    if (prod.ph >= a.n_phases) return;
    uint8_t* dst = ring + (size_t)slot * a.ring_stride;
    if (prod.sub == 1) {  // n whole down tiles of the CTA's nj groups: one copy per group (group-major units)
      const int n = min(max(1, GPC / prod.nj), prod.end - prod.u);
      const uint32_t gbytes = (uint32_t)(n * GB);
      mbar_arrive_expect_tx(&wb[slot], (uint32_t)prod.nj * gbytes);
      for (int jj = 0; jj < prod.nj; ++jj)
        bulk_g2s(dst + (size_t)jj * gbytes, prod.blob + ((int64_t)(prod.j0 + jj) * prod.G + prod.u) * GB, gbytes,
                 &wb[slot]);
      ++issued;
      prod.u += n;
      if (prod.u >= prod.end) set_phase(prod, prod.ph + 1);
      return;
    }
    const int gb = EXT ? prod.gb : GB;
    const int n = min(min(EXT ? prod.gpc : GPC, prod.end - prod.u), prod.G - prod.gi);  // never crosses a row tile
    mbar_arrive_expect_tx(&wb[slot], (uint32_t)(n * gb));
    bulk_g2s(dst, prod.blob + (int64_t)prod.u * gb, (uint32_t)(n * gb), &wb[slot]);
    ++issued;
    prod.u += n;
    prod.gi += n;
    if (prod.gi == prod.G) prod.gi = 0;
    if (prod.u >= prod.end) {
      if (phs[prod.ph].kind == PD_FFN && set_down(prod, prod.ph)) return;
      set_phase(prod, prod.ph + 1);
    }
  };
  if (lane == 0) {
    set_phase(prod, 0);
    for (int r = 0; r < PD_RING; ++r) issue_next(r);
  }
  if (tid == PD_KV_T && has_item) {
    const int ph = next_attn(0);
    if (ph < a.n_phases) kv_issue(ph, pg0);
  }

  // A warp whose copy wait runs out stops consuming and raises the abort flag;
  // every CTA then leaves at its next grid barrier (a CTA-uniform decision).
  bool wfail = false;
  int bar_k = 0, attn_idx = 0;
  const int xep = EXT && a.tp_size > 1 ? *reinterpret_cast<volatile int*>(a.xepoch) : 0;  // this launch's number
  for (int ph = 0; ph < a.n_phases; ++ph) {
    const PdPhase& P = phs[ph];
    if ((P.kind == PD_GEMV || P.kind == PD_FFN) && P.norm_w)  // constant: pull this thread's norm weights into L1 before the wait
      for (int i = tid; i < (P.cols >> 2); i += PD_THREADS) {
        const float* p = P.norm_w + (i >> 2) * 16 + 2 * (i & 3);
        asm volatile("prefetch.global.L1 [%0];" :: "l"(p));
        asm volatile("prefetch.global.L1 [%0];" :: "l"(p + 8));
      }
    unsigned long long* t_arr = a.trace ? a.trace + ((size_t)PD_TRACE_ROWS * ph) * NC + cta : nullptr;
    if (ph > 0 && !(EXT && P.xbar ? pd_xbarrier(a, xep, P.xbar, flag, t_arr) : pd_barrier(a, ++bar_k, flag, t_arr)))
      break;
    // trace marks of this phase: row PD_TRACE_ROWS ph + 1 departure, + 2 and + 3 the marks below; the
    // previous phase's chunk-wait sums (complete: every warp has passed the barrier) go to its rows + 4, + 5
    unsigned long long* t_mark =
        a.trace && tid == PD_SYNC_T ? a.trace + ((size_t)PD_TRACE_ROWS * ph + 1) * NC + cta : nullptr;
    if (t_mark) {
      *t_mark = gtimer();
      if (ph > 0) {
        unsigned long long* prev = a.trace + ((size_t)PD_TRACE_ROWS * (ph - 1)) * NC + cta;
        prev[4 * NC] = wacc[0];
        prev[5 * NC] = wacc[1];
      }
      wacc[0] = wacc[1] = 0ull;
    }

    if (P.kind == PD_ATTN) {
      if (has_item) {
        __half* q_h = reinterpret_cast<__half*>(work);                              // [PD_MAXG][HD + 8]
        float* sc = reinterpret_cast<float*>(work + (size_t)PD_MAXG * (HD + 8) * 2);  // [PD_MAXG][PD_PAGE]
        float* ml = sc + PD_MAXG * PD_PAGE;           // [PD_MAXG][4]: m, l, alpha, den
        const float* cs = a.cos_t + (int64_t)sp.pos * H2;
        const float* sn = a.sin_t + (int64_t)sp.pos * H2;
        // O accumulator fragment: warp w < HD/8 owns dims [8w, 8w+8); row g = query head g
        float oc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int pg = pg0; pg < pg1; ++pg) {
          if (tid == PD_KV_T) {
            if (pg > pg0) kv_issue(ph, pg);
            const bool okw = wait_bar(kvbar, (uint32_t)(kv_waited & 1));
            ++kv_waited;
            if (!okw) { atomicExch(&a.sync[2], 1); atomicExch(a.err, DEV_ERR_TIMEOUT); }
          }
          __syncthreads();
          const int t0 = pg * PD_PAGE, n = min(PD_PAGE, sp.L - t0);
          // one batch of loads: the queries and, in the split holding it, the new
          // token's k and v; then RoPE (queries pre-scaled, fp16, rows >= GQ zero),
          // k and v to the page and the cache
          {
            constexpr int QI = (PD_MAXG * HD + PD_THREADS - 1) / PD_THREADS;
            const bool first = pg == pg0, kv_here = t0 <= sp.pos && sp.pos < t0 + PD_PAGE && tid < HD;
            float qa[QI], qb[QI], qc[QI], qs[QI];
#pragma unroll
            for (int r = 0; r < QI; ++r) {
              const int i = tid + r * PD_THREADS, j = i / HD, dd = i - j * HD, j0 = dd < H2 ? dd : dd - H2;
              qa[r] = qb[r] = qc[r] = qs[r] = 0.f;
              if (first && i < PD_MAXG * HD && j < GQ) {
                const float* qh = a.qkv + (int64_t)(kvh * GQ + j) * HD;
                qa[r] = __ldcg(qh + j0); qb[r] = __ldcg(qh + j0 + H2); qc[r] = cs[j0]; qs[r] = sn[j0];
              }
            }
            const int kd = tid < HD ? tid : 0, kj0 = kd < H2 ? kd : kd - H2;
            float ka = 0.f, kb = 0.f, kc = 0.f, ks = 0.f, vv = 0.f;
            if (kv_here) {
              const float* kh = a.qkv + (int64_t)(d.n_heads + kvh) * HD;
              const float* vh = a.qkv + (int64_t)(d.n_heads + d.n_kv + kvh) * HD;
              ka = __ldcg(kh + kj0); kb = __ldcg(kh + kj0 + H2); kc = cs[kj0]; ks = sn[kj0]; vv = __ldcg(vh + kd);
            }
            if (first) {
#pragma unroll
              for (int r = 0; r < QI; ++r) {
                const int i = tid + r * PD_THREADS, j = i / HD, dd = i - j * HD;
                if (i < PD_MAXG * HD)
                  q_h[j * (HD + 8) + dd] = __float2half_rn(
                      (dd < H2 ? qa[r] * qc[r] - qb[r] * qs[r] : qb[r] * qc[r] + qa[r] * qs[r]) * d.scale);
              }
              if (tid < GQ) { ml[tid * 4 + 0] = -INFINITY; ml[tid * 4 + 1] = 0.f; }
            }
            if (kv_here) {
              const int r = sp.pos - t0;
              const int64_t off = (((int64_t)a.block_table[pg] * d.n_kv + kvh) * PD_PAGE + r) * HD;
              const __half kq = __float2half_rn(kd < H2 ? ka * kc - kb * ks : kb * kc + ka * ks);
              const __half vq = __float2half_rn(vv);
              Ks[r * HD + kd] = kq;
              Vs[r * HD + kd] = vq;
              P.kv.k_pages[off + kd] = kq;
              P.kv.v_pages[off + kd] = vq;
            }
          }
          for (int i = tid; i < (PD_PAGE - n) * (HD / 8); i += PD_THREADS)  // V rows past the context: 0
            reinterpret_cast<uint4*>(Vs + n * HD)[i] = make_uint4(0u, 0u, 0u, 0u);
          __syncthreads();
          if (warp < PD_PAGE / 8) {  // S = Q K^T on the tensor cores: warp w scores positions [8w, 8w+8)
            float c4[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t* q32 = reinterpret_cast<const uint32_t*>(q_h + g * (HD + 8));
            const uint32_t* k32 = reinterpret_cast<const uint32_t*>(Ks + (warp * 8 + g) * HD);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks)
              mma16816(c4, q32[ks * 8 + tq], 0u, q32[ks * 8 + 4 + tq], 0u, k32[ks * 8 + tq], k32[ks * 8 + 4 + tq]);
            if (g < GQ) *reinterpret_cast<float2*>(sc + g * PD_PAGE + warp * 8 + 2 * tq) = make_float2(c4[0], c4[1]);
          }
          __syncthreads();
          if (warp < GQ) {  // online softmax, one warp per query head
            const int j = warp;
            const float v0 = lane < n ? sc[j * PD_PAGE + lane] : -INFINITY;
            const float v1 = lane + 32 < n ? sc[j * PD_PAGE + lane + 32] : -INFINITY;
            const float m_old = ml[j * 4 + 0];
            const float m_new = fmaxf(m_old, warp_max(fmaxf(v0, v1)));
            const float e0 = lane < n ? __expf(v0 - m_new) : 0.f;
            const float e1 = lane + 32 < n ? __expf(v1 - m_new) : 0.f;
            const float sum = warp_sum(e0 + e1);
            const float alpha = m_old == -INFINITY ? 0.f : __expf(m_old - m_new);
            sc[j * PD_PAGE + lane] = e0;
            sc[j * PD_PAGE + lane + 32] = e1;
            __syncwarp();
            if (lane == 0) { ml[j * 4 + 0] = m_new; ml[j * 4 + 1] = ml[j * 4 + 1] * alpha + sum; ml[j * 4 + 2] = alpha; }
          }
          __syncthreads();
          if (warp < HD / 8) {  // O = alpha O + P V on the tensor cores (P in fp16, rows >= GQ zero)
            const bool row = g < GQ;
            const float al = row ? ml[g * 4 + 2] : 0.f;
            oc[0] *= al; oc[1] *= al;
            const float* pr = sc + (row ? g : 0) * PD_PAGE;
            const __half* vc = Vs + warp * 8 + g;
#pragma unroll
            for (int ks = 0; ks < PD_PAGE / 16; ++ks) {
              const int k0 = ks * 16 + 2 * tq;
              const float2 p0 = *reinterpret_cast<const float2*>(pr + k0);
              const float2 p1 = *reinterpret_cast<const float2*>(pr + k0 + 8);
              const uint32_t a0 = row ? h2u(__floats2half2_rn(p0.x, p0.y)) : 0u;
              const uint32_t a2 = row ? h2u(__floats2half2_rn(p1.x, p1.y)) : 0u;
              const uint32_t b0 = h2u(__halves2half2(vc[k0 * HD], vc[(k0 + 1) * HD]));
              const uint32_t b1 = h2u(__halves2half2(vc[(k0 + 8) * HD], vc[(k0 + 9) * HD]));
              mma16816(oc, a0, 0u, a2, 0u, b0, b1);
            }
          }
          __syncthreads();
        }
        // this split's partial: o [GQ][HD] and (m, l) per query head
        const int item = kvh * sp.ns + split;
        float* part_o = a.attn_part + (size_t)item * GQ * HD;
        float* part_ml = a.attn_part + (size_t)d.n_kv * a.max_split * GQ * HD + (size_t)item * GQ * 2;
        if (warp < HD / 8 && g < GQ) *reinterpret_cast<float2*>(part_o + g * HD + warp * 8 + 2 * tq) = make_float2(oc[0], oc[1]);
        if (tid < GQ) *reinterpret_cast<float2*>(part_ml + tid * 2) = make_float2(ml[tid * 4 + 0], ml[tid * 4 + 1]);
        // wait for every split of this KV head (co-resident CTAs, bounded wait)
        __syncthreads();
        if (t_mark) t_mark[NC] = gtimer();  // this split's partial is written
        if (tid == PD_SYNC_T) {
          asm volatile("red.release.gpu.global.add.s32 [%0], 1;" :: "l"(a.attn_cnt + kvh) : "memory");
          flag[1] = pd_wait_count(a, a.attn_cnt + kvh, sp.ns * (attn_idx + 1));
        }
        __syncthreads();
        if (t_mark) t_mark[2 * NC] = gtimer();  // every split of the head has published
        if (flag[1]) {
          // this split merges outputs [o_lo, o_hi) of its head group (GQ*HD values): one batch of loads
          const int no = GQ * HD, o_lo = split * no / sp.ns, o_hi = (split + 1) * no / sp.ns;
          const int nout = o_hi - o_lo, j_lo = o_lo / HD, nj = (o_hi - 1) / HD - j_lo + 1;
          float* mv = ml + PD_MAXG * 4;                 // [nj][ns] (nj*ns <= GQ + 2 ns): m, then weight
          float* lv = mv + 4 * PD_MAXSPLIT;             // [nj][ns]
          float* ov = lv + 4 * PD_MAXSPLIT;             // [nout][ns] (<= GQ*HD + ns)
          const float* base_o = a.attn_part + (size_t)kvh * sp.ns * GQ * HD;
          const float* base_ml = a.attn_part + (size_t)d.n_kv * a.max_split * GQ * HD + (size_t)kvh * sp.ns * GQ * 2;
          {  // one batch of loads (nj * ns <= PD_MAXG * PD_MAXSPLIT = PD_THREADS; nout * ns bounded below)
            constexpr int MAXI = (PD_MAXG * HD + PD_MAXSPLIT + PD_THREADS - 1) / PD_THREADS;
            float2 mlv = make_float2(0.f, 0.f);
            const bool has_ml = tid < nj * sp.ns;
            if (has_ml) {
              const int jj = tid / sp.ns, s2 = tid - jj * sp.ns;
              mlv = __ldcg(reinterpret_cast<const float2*>(base_ml + ((size_t)s2 * GQ + j_lo + jj) * 2));
            }
            float ovr[MAXI];
#pragma unroll
            for (int r = 0; r < MAXI; ++r) {
              const int i = tid + r * PD_THREADS;
              ovr[r] = 0.f;
              if (i < nout * sp.ns) {
                const int oo = i / sp.ns, s2 = i - oo * sp.ns;
                ovr[r] = __ldcg(base_o + (size_t)s2 * GQ * HD + o_lo + oo);
              }
            }
            if (has_ml) { mv[tid] = mlv.x; lv[tid] = mlv.y; }
#pragma unroll
            for (int r = 0; r < MAXI; ++r)
              if (tid + r * PD_THREADS < nout * sp.ns) ov[tid + r * PD_THREADS] = ovr[r];
          }
          __syncthreads();
          // warp jj < nj: split weights e^(m_s - M) of query head j_lo + jj and their
          // denominator; lanes stride over the splits, fixed-order warp reductions
          if (warp < nj) {
            float M = -INFINITY;
            for (int s2 = lane; s2 < sp.ns; s2 += 32) M = fmaxf(M, mv[warp * sp.ns + s2]);
            M = warp_max(M);
            float den = 0.f;
            for (int s2 = lane; s2 < sp.ns; s2 += 32) {
              const float m = mv[warp * sp.ns + s2];
              const float w = m == -INFINITY ? 0.f : __expf(m - M);
              mv[warp * sp.ns + s2] = w;
              den = fmaf(w, lv[warp * sp.ns + s2], den);
            }
            den = warp_sum(den);
            if (lane == 0) ml[warp * 4 + 3] = den;
          }
          __syncthreads();
          for (int oo = warp; oo < nout; oo += PD_WARPS) {  // one warp per output, lanes over splits
            const int o = o_lo + oo, jj = o / HD - j_lo;
            float num = 0.f;
            for (int s2 = lane; s2 < sp.ns; s2 += 32) num = fmaf(mv[jj * sp.ns + s2], ov[oo * sp.ns + s2], num);
            num = warp_sum(num);
            if (lane == 0) a.attn_out[(int64_t)kvh * no + o] = num / (ml[jj * 4 + 3] + 1e-9f);
          }
        }
        // the page buffer is free: start copying this CTA's page of the next layer
        if (tid == PD_KV_T) {
          const int nph = next_attn(ph + 1);
          if (nph < a.n_phases) kv_issue(nph, pg0);
        }
      }
      ++attn_idx;
      continue;
    }

    // ========================= GEMV (FFN: gate|up part) =========================
    const int K = P.cols, G = P.G;
    int t0, t1;
    pd_tiles(P, cta, NC, KPG, t0, t1);
    const int c0 = t0 * G, c1 = t1 * G;
    if (tid <= PD_WARPS) wr[tid] = pd_rng(c0, c1, tid, PD_WARPS);  // read after the prologue's barrier
    const bool has_add = P.epi == PD_EPI_RESID || P.bias;
    uint4* xf = reinterpret_cast<uint4*>(work);                     // [ks_n/2][4 tq] x 2 k-steps
    float* sx = reinterpret_cast<float*>(work + (size_t)K * 2);     // [G] (+8 pad)
    {
      // one batch of loads: x (and norm weights), this CTA's residual / bias rows
      if (has_add) {
        const int r0 = t0 * 16, r1 = min(t1 * 16, P.rows);
        const bool fold = P.epi == PD_EPI_RESID && P.acc;  // h + acc is the residual; clear acc
        for (int r = r0 + tid; r < r1; r += PD_THREADS) {
          float h = P.epi == PD_EPI_RESID ? __ldcg(P.y + r) : 0.f;
          if (fold) {
            h += __ll2float_rn((long long)__ldcg(P.acc + r)) * PD_UNFIX;
            P.acc[r] = 0ull;
          }
          addv[r - r0] = h + (P.bias ? P.bias[r] : 0.f);
        }
      }
      // x = h + acc (an FFN phase's acc is its own output, not an input)
      const unsigned long long* xacc = P.kind == PD_GEMV && P.epi != PD_EPI_RESID ? P.acc : nullptr;
      // x -> (RMS-normalised) fp16 B fragments and per-group sums of the fp16 x.
      // A group's KPG*4 items are consecutive, so for KPG <= 8 they sit in one
      // warp (or half-warp) and Sx is a shuffle reduction of the rounded values.
      const int items = K >> 2;  // (k-step, tq) items of 4 values: k, k+1, k+8, k+9
      uint2* xf2 = reinterpret_cast<uint2*>(xf);
      auto put = [&](int i, float v0, float v1, float v2, float v3) {
        const int s = i >> 2, tqi = i & 3;
        const __half2 h01 = __floats2half2_rn(v0, v1), h23 = __floats2half2_rn(v2, v3);
        xf2[(((s >> 1) * 4 + tqi) << 1) + (s & 1)] = make_uint2(h2u(h01), h2u(h23));
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        return (f01.x + f01.y) + (f23.x + f23.y);
      };
      auto group_sum = [&](int i, float v) {  // all 32 lanes; lane 0 of the group writes
        if constexpr (KPG <= 8) {
#pragma unroll
          for (int o = KPG * 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if ((lane & (KPG * 4 - 1)) == 0 && i < items) sx[i / (KPG * 4)] = v;
        }
      };
      if (P.norm_w) {  // K <= PD_KNORM: the row stays in registers across the reduction
        float xv[PD_NREG][4];
        float ss = 0.f;
        if (EXT && P.xsum) {  // tensor parallel: x = h + every rank's partial sums, added in rank order
          const float* rb = a.xrecv_local + (int64_t)P.xpar * a.tp_size * a.xcap;
#pragma unroll
          for (int j = 0; j < PD_NREG; ++j) {
            const int i = tid + j * PD_THREADS;
            xv[j][0] = xv[j][1] = xv[j][2] = xv[j][3] = 0.f;
            if (i < items) {
              const int k = (i >> 2) * 16 + 2 * (i & 3);
              const float2 v0 = __ldcg(reinterpret_cast<const float2*>(P.x + k));
              const float2 v1 = __ldcg(reinterpret_cast<const float2*>(P.x + k + 8));
              xv[j][0] = v0.x; xv[j][1] = v0.y; xv[j][2] = v1.x; xv[j][3] = v1.y;
            }
          }
          for (int r = 0; r < a.tp_size; r += 2) {  // two ranks' loads in one batch
            const bool two = r + 1 < a.tp_size;
            const float* r0p = rb + (int64_t)r * a.xcap;
            const float* r1p = r0p + a.xcap;
            float2 u[PD_NREG][4];
#pragma unroll
            for (int j = 0; j < PD_NREG; ++j) {
              const int i = tid + j * PD_THREADS;
              const int k = (i >> 2) * 16 + 2 * (i & 3);
              u[j][0] = u[j][1] = u[j][2] = u[j][3] = make_float2(0.f, 0.f);
              if (i < items) {
                u[j][0] = __ldcg(reinterpret_cast<const float2*>(r0p + k));
                u[j][1] = __ldcg(reinterpret_cast<const float2*>(r0p + k + 8));
                if (two) {
                  u[j][2] = __ldcg(reinterpret_cast<const float2*>(r1p + k));
                  u[j][3] = __ldcg(reinterpret_cast<const float2*>(r1p + k + 8));
                }
              }
            }
#pragma unroll
            for (int j = 0; j < PD_NREG; ++j) {
              xv[j][0] += u[j][0].x; xv[j][1] += u[j][0].y; xv[j][2] += u[j][1].x; xv[j][3] += u[j][1].y;
              if (two) { xv[j][0] += u[j][2].x; xv[j][1] += u[j][2].y; xv[j][2] += u[j][3].x; xv[j][3] += u[j][3].y; }
            }
          }
          // the new residual: this CTA's share of the rows goes to the other buffer
          const int o0 = pd_rng(0, K, cta, NC), o1 = pd_rng(0, K, cta + 1, NC);
#pragma unroll
          for (int j = 0; j < PD_NREG; ++j) {
            const int i = tid + j * PD_THREADS;
            if (i < items) {
              const int k = (i >> 2) * 16 + 2 * (i & 3);
              if (P.h_out) {
                if (k >= o0 && k < o1) P.h_out[k] = xv[j][0];
                if (k + 1 >= o0 && k + 1 < o1) P.h_out[k + 1] = xv[j][1];
                if (k + 8 >= o0 && k + 8 < o1) P.h_out[k + 8] = xv[j][2];
                if (k + 9 >= o0 && k + 9 < o1) P.h_out[k + 9] = xv[j][3];
              }
              ss += xv[j][0] * xv[j][0] + xv[j][1] * xv[j][1] + xv[j][2] * xv[j][2] + xv[j][3] * xv[j][3];
            }
          }
        } else {
#pragma unroll
        for (int j = 0; j < PD_NREG; ++j) {
          const int i = tid + j * PD_THREADS;
          if (i < items) {
            const int k = (i >> 2) * 16 + 2 * (i & 3);
            const float2 v0 = __ldcg(reinterpret_cast<const float2*>(P.x + k));
            const float2 v1 = __ldcg(reinterpret_cast<const float2*>(P.x + k + 8));
            xv[j][0] = v0.x; xv[j][1] = v0.y; xv[j][2] = v1.x; xv[j][3] = v1.y;
            if (xacc) {
              const ulonglong2 a0 = __ldcg(reinterpret_cast<const ulonglong2*>(xacc + k));
              const ulonglong2 a1 = __ldcg(reinterpret_cast<const ulonglong2*>(xacc + k + 8));
              xv[j][0] += __ll2float_rn((long long)a0.x) * PD_UNFIX;
              xv[j][1] += __ll2float_rn((long long)a0.y) * PD_UNFIX;
              xv[j][2] += __ll2float_rn((long long)a1.x) * PD_UNFIX;
              xv[j][3] += __ll2float_rn((long long)a1.y) * PD_UNFIX;
            }
            ss += xv[j][0] * xv[j][0] + xv[j][1] * xv[j][1] + xv[j][2] * xv[j][2] + xv[j][3] * xv[j][3];
          }
        }
        }
        const float inv = rsqrtf(block_sum(ss, red) / K + a.eps);
#pragma unroll
        for (int j = 0; j < PD_NREG; ++j) {
          const int i = tid + j * PD_THREADS;
          float sv = 0.f;
          if (i < items) {  // norm weights were prefetched into L1 before the barrier
            const int k = (i >> 2) * 16 + 2 * (i & 3);
            const float2 n0 = *reinterpret_cast<const float2*>(P.norm_w + k);
            const float2 n1 = *reinterpret_cast<const float2*>(P.norm_w + k + 8);
            sv = put(i, xv[j][0] * inv * n0.x, xv[j][1] * inv * n0.y, xv[j][2] * inv * n1.x, xv[j][3] * inv * n1.y);
          }
          if (j * PD_THREADS < items) group_sum(i, sv);
        }
      } else {
#pragma unroll 4
        for (int b = 0; b < items; b += PD_THREADS) {
          const int i = b + tid;
          float sv = 0.f;
          if (i < items) {
            const int k = (i >> 2) * 16 + 2 * (i & 3);
            float2 v0 = __ldcg(reinterpret_cast<const float2*>(P.x + k));
            float2 v1 = __ldcg(reinterpret_cast<const float2*>(P.x + k + 8));
            if (xacc) {
              const ulonglong2 a0 = __ldcg(reinterpret_cast<const ulonglong2*>(xacc + k));
              const ulonglong2 a1 = __ldcg(reinterpret_cast<const ulonglong2*>(xacc + k + 8));
              v0.x += __ll2float_rn((long long)a0.x) * PD_UNFIX;
              v0.y += __ll2float_rn((long long)a0.y) * PD_UNFIX;
              v1.x += __ll2float_rn((long long)a1.x) * PD_UNFIX;
              v1.y += __ll2float_rn((long long)a1.y) * PD_UNFIX;
            }
            sv = put(i, v0.x, v0.y, v1.x, v1.y);
          }
          group_sum(i, sv);
        }
      }
      __syncthreads();
      if (KPG > 8) {  // a group spans two warps: sum its fp16 x from shared memory
        for (int grp = tid; grp < G; grp += PD_THREADS) {
          const uint4* src = xf + (size_t)grp * (KPG >> 1) * 4;
          float v = 0.f;
#pragma unroll 4
          for (int e = 0; e < KPG * 2; ++e) {
            const uint4 u = src[e];
            const float2 f0 = __half22float2(u2h(u.x)), f1 = __half22float2(u2h(u.y));
            const float2 f2 = __half22float2(u2h(u.z)), f3 = __half22float2(u2h(u.w));
            v += ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
          }
          sx[grp] = v;
        }
        __syncthreads();
      }
    }

    if (t_mark) t_mark[NC] = gtimer();  // prologue done: x fragments and group sums in shared memory

    // epilogue of the 16 rows of tile t (all 32 lanes; lane r < 16 holds row t*16 + r)
    auto tile_out = [&](int t, float v) {
      const int row = t * 16 + lane;
      const bool in = lane < 16 && row < P.rows;
      if (in && has_add) v += addv[row - t0 * 16];
      if (P.epi == PD_EPI_SWIGLU) {
        const float up = __shfl_down_sync(0xffffffffu, v, 1);
        if (in && !(lane & 1)) {
          const float m = (v / (1.0f + expf(-v))) * up;
          if (P.kind == PD_FFN) mloc[(row >> 1) - t0 * 8] = m;
          else P.y[row >> 1] = m;
        }
      } else if (EXT && P.epi == PD_EPI_XPUSH) {  // this rank's partial sum of the row into every rank's slot
        if (in) {
          const int64_t off = ((int64_t)P.xpar * a.tp_size + a.tp_rank) * a.xcap + row;
#pragma unroll
          for (int r = 0; r < PD_MAX_RANKS; ++r)
            if (r < a.tp_size) a.xrecv[r][off] = v;
        }
      } else if (in) {
        P.y[row] = v;
      }
    };

    const int w0 = wr[warp], w1 = wr[warp + 1];
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    int t = w0 / G, gi = w0 - t * G;  // current row tile, group within it
    const int uprec = EXT ? (P.prec == 0 ? 4 : P.prec) : 4;
    const int ugpc = uprec == 4 ? GPC : uprec == 8 ? a.ring_stride / PD_UNIT8 : a.ring_stride / PD_UNIT16;
    for (int u = w0; u < w1 && !wfail;) {
      const int n = min(min(ugpc, w1 - u), G - gi);
      const int slot = consumed % PD_RING;
      int okl = 0;
      if (lane == 0) {
        const uint64_t tw = a.trace ? gtimer() : 0;
        okl = wait_bar(&wb[slot], (uint32_t)((consumed / PD_RING) & 1));
        if (a.trace) atomicAdd(&wacc[0], (unsigned long long)(gtimer() - tw));
      }
      if (!__shfl_sync(0xffffffffu, okl, 0)) {
        if (lane == 0) { atomicExch(&a.sync[2], 1); atomicExch(a.err, DEV_ERR_TIMEOUT); }
        wfail = true;
        break;
      }
      const uint8_t* buf = ring + (size_t)slot * a.ring_stride;
      const uint4* xb[1] = {xf + gi * KPG * 2 + tq};
      const float* sxg = sx + gi;
      if (EXT && uprec != 4) {
        for (int gr = 0; gr < n; ++gr) {
          if (uprec == 8) pd_unit_i8<KPG>(buf + gr * PD_UNIT8, lane, xb[0] + gr * KPG * 2, sxg[gr], acc[0][0], acc[0][2]);
          else pd_unit_f16<KPG>(buf + gr * PD_UNIT16, lane, xb[0] + gr * KPG * 2, acc[0][0], acc[0][2]);
        }
      } else if (n == GPC) {
        mma_chunk<KPG, 1, GPC, true, 1>(buf, lane, xb, sxg, acc);
      } else {
        for (int gr = 0; gr < n; ++gr) {
          const uint4* xg[1] = {xb[0] + gr * KPG * 2};
          mma_chunk<KPG, 1, 1, true, 1>(buf + gr * GB, lane, xg, sxg + gr, acc);
        }
      }
      ++consumed;
      __syncwarp();
      if (lane == 0) issue_next(slot);
      u += n;
      gi += n;
      if (u < w1 && gi < G) continue;
      // ---- this warp's part of row tile tt is complete ----
      const int tt = t;
      if (gi == G) { gi = 0; ++t; }
      const int tu0 = tt * G, tu1 = tu0 + G;
      const int side = (tt == w0 / G) ? 0 : 1;
      float* mine = wpart + (warp * 2 + side) * 16;
      if (tq == 0) { mine[g] = acc[0][0]; mine[g + 8] = acc[0][2]; }
      acc[0][0] = acc[0][1] = acc[0][2] = acc[0][3] = 0.f;
      __syncwarp();
      if (w0 <= tu0 && tu1 <= w1) {  // the warp owns the whole tile
        tile_out(tt, lane < 16 ? mine[lane] : 0.f);
        __syncwarp();
        continue;
      }
      // shared with other warps of the CTA: the last contributor sums them in warp order
      int wa = warp, wz = warp;  // warps whose ranges meet the tile (wr[] is ascending)
      while (wa > 0 && wr[wa] > tu0) --wa;
      while (wz < PD_WARPS - 1 && wr[wz + 1] < tu1) ++wz;
      int contrib = 0;
      for (int w = wa; w <= wz; ++w) contrib += wr[w] < wr[w + 1];
      __threadfence_block();
      int last = 0;
      if (lane == 0) last = atomicAdd(&wcnt[wa], 1) == contrib - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      if (lane == 0) wcnt[wa] = 0;
      __threadfence_block();
      float v = 0.f;
      if (lane < 16)
        for (int w = wa; w <= wz; ++w) {
          const int ws0 = wr[w];
          if (ws0 == wr[w + 1]) continue;
          const int sd = (tt == ws0 / G) ? 0 : 1;
          v += *reinterpret_cast<volatile float*>(wpart + (w * 2 + sd) * 16 + lane);
        }
      tile_out(tt, v);
    }
    if (P.kind != PD_FFN) continue;

    // ============ FFN: down_proj partial sums over this CTA's channels ============
    __syncthreads();  // every SwiGLU channel of the CTA is in mloc
    if (t_mark) t_mark[2 * NC] = gtimer();  // gate|up done
    const int j0 = pd_rng(0, P.G2, cta, NC), nj = pd_rng(0, P.G2, cta + 1, NC) - j0;
    if (nj == 0) continue;
    {
      const int items = nj * KPG * 4;  // (k-step, tq) items of the nj groups
      uint2* xf2 = reinterpret_cast<uint2*>(xf);
      // a group's KPG*4 items sit in one warp (or half-warp) for KPG <= 8: its Sx is a
      // shuffle reduction of the rounded values (no serial pass over shared memory)
      for (int i0 = 0; i0 < items; i0 += PD_THREADS) {
        const int i = i0 + tid;
        float v = 0.f;
        if (i < items) {
          const int s = i >> 2, tqi = i & 3, k = s * 16 + 2 * tqi;
          const __half2 h01 = __floats2half2_rn(mloc[k], mloc[k + 1]);
          const __half2 h23 = __floats2half2_rn(mloc[k + 8], mloc[k + 9]);
          xf2[(((s >> 1) * 4 + tqi) << 1) + (s & 1)] = make_uint2(h2u(h01), h2u(h23));
          const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
          v = (f01.x + f01.y) + (f23.x + f23.y);
        }
        if constexpr (KPG <= 8) {
#pragma unroll
          for (int o = KPG * 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if ((lane & (KPG * 4 - 1)) == 0 && i < items) sx[i / (KPG * 4)] = v;
        }
      }
      __syncthreads();
      if constexpr (KPG > 8) {  // a group spans two warps: sum its fp16 x from shared memory
        for (int grp = tid; grp < nj; grp += PD_THREADS) {
          const uint4* src = xf + (size_t)grp * (KPG >> 1) * 4;
          float v = 0.f;
          for (int e = 0; e < KPG * 2; ++e) {
            const uint4 u = src[e];
            const float2 f0 = __half22float2(u2h(u.x)), f1 = __half22float2(u2h(u.y));
            const float2 f2 = __half22float2(u2h(u.z)), f3 = __half22float2(u2h(u.w));
            v += ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
          }
          sx[grp] = v;
        }
        __syncthreads();
      }
    }
    const int Td = (P.rows2 + 15) >> 4;
    const int d0 = pd_rng(0, Td, warp, PD_WARPS), d1 = pd_rng(0, Td, warp + 1, PD_WARPS);
    const int per = max(1, GPC / nj);  // whole tiles per chunk
    // fixed-point sums (order-independent); all 32 lanes call it: lane tq 0 adds row g,
    // lane tq 1 row g + 8 (handed over by a shuffle), so one conversion and one atomic per lane
    auto put_rows = [&](int t, float r_g, float r_g8) {
      const float v8 = __shfl_up_sync(0xffffffffu, r_g8, 1);
      const int r = t * 16 + g + (tq == 1 ? 8 : 0);
      if (tq < 2 && r < P.rows2)
        atomicAdd(P.acc + r, (unsigned long long)__float2ll_rn((tq == 0 ? r_g : v8) * PD_FIX));
    };
    for (int u = d0; u < d1 && !wfail;) {
      const int n = min(per, d1 - u);
      const int slot = consumed % PD_RING;
      int okl = 0;
      if (lane == 0) {
        const uint64_t tw = a.trace ? gtimer() : 0;
        okl = wait_bar(&wb[slot], (uint32_t)((consumed / PD_RING) & 1));
        if (a.trace) atomicAdd(&wacc[1], (unsigned long long)(gtimer() - tw));
      }
      if (!__shfl_sync(0xffffffffu, okl, 0)) {
        if (lane == 0) { atomicExch(&a.sync[2], 1); atomicExch(a.err, DEV_ERR_TIMEOUT); }
        wfail = true;
        break;
      }
      const uint8_t* buf = ring + (size_t)slot * a.ring_stride;
      if (nj == 1 && n == GPC) {
        float acc4[GPC][4];
#pragma unroll
        for (int i = 0; i < GPC; ++i) acc4[i][0] = acc4[i][1] = acc4[i][2] = acc4[i][3] = 0.f;
        mma_units<KPG, GPC>(buf, lane, xf + tq, sx[0], acc4);
#pragma unroll
        for (int i = 0; i < GPC; ++i) put_rows(u + i, acc4[i][0], acc4[i][2]);
      } else {
        for (int i = 0; i < n; ++i) {
          float acc1[1][4] = {{0.f, 0.f, 0.f, 0.f}};
          for (int jj = 0; jj < nj; ++jj) {
            const uint4* xg[1] = {xf + jj * KPG * 2 + tq};
            mma_chunk<KPG, 1, 1, true, 1>(buf + (size_t)(jj * n + i) * GB, lane, xg, sx + jj, acc1);
          }
          put_rows(u + i, acc1[0][0], acc1[0][2]);
        }
      }
      ++consumed;
      __syncwarp();
      if (lane == 0) issue_next(slot);
      u += n;
    }
  }

  if (a.trace) {  // end of this CTA's last phase
    __syncthreads();
    if (tid == PD_SYNC_T) {
      unsigned long long* last = a.trace + ((size_t)PD_TRACE_ROWS * (a.n_phases - 1)) * NC + cta;
      last[4 * NC] = wacc[0];
      last[5 * NC] = wacc[1];
      a.trace[((size_t)PD_TRACE_ROWS * a.n_phases) * NC + cta] = gtimer();
    }
  }
  // copies still in flight (abort path) are waited for, bounded, before exit
  if (lane == 0)
    for (int q = consumed; q < issued; ++q) wait_bar(&wb[q % PD_RING], (uint32_t)((q / PD_RING) & 1));
  if (tid == PD_KV_T)
    for (; kv_waited < kv_uses; ++kv_waited) wait_bar(kvbar, (uint32_t)(kv_waited & 1));
  __syncthreads();
  if (tid == PD_SYNC_T) {  // the last CTA out resets the counters and the FFN accumulator for the next launch
    __threadfence();
    flag[2] = atomicAdd(&a.sync[1], 1) == NC - 1;
  }
  __syncthreads();
  if (flag[2]) {
    for (int i = tid; i < a.acc_n; i += PD_THREADS) a.acc[i] = 0ull;
    if (tid == PD_SYNC_T) {
      if (EXT && a.tp_size > 1) *a.xepoch = xep + 1;
      for (int h = 0; h < d.n_kv; ++h) a.attn_cnt[h] = 0;
      a.sync[0] = 0;
      a.sync[2] = 0;
      __threadfence();
      a.sync[1] = 0;
    }
  }
}

template <int KPG, int HD, bool EXT>
static int persist_setup(const PdPlan& plan, bool launch, cudaStream_t st, int* max_blocks) {
  auto kern = persist_decode_kernel<KPG, HD, EXT>;
  if (int rc = smem_attr_once<persist_decode_kernel<KPG, HD, EXT>>(227 * 1024)) return rc;
  if (max_blocks) N730_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(max_blocks, kern, PD_THREADS, plan.smem));
  if (!launch) return N730_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(PD_THREADS);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  N730_CUDA(cudaLaunchKernelEx(&cfg, kern, plan.a));
  return N730_OK;
}

static int persist_dispatch(const PdPlan& plan, int head_dim, bool launch, cudaStream_t st, int* max_blocks) {
  const int kpg = plan.a.kpg;
  if (plan.a.tp_size > 1 || plan.a.tab_off < 0 || plan.a.mixed) {  // EXT features: group 128 only
    if (kpg != 8) return N730_UNSUPPORTED;
    if (head_dim == 128) return persist_setup<8, 128, true>(plan, launch, st, max_blocks);
    return persist_setup<8, 64, true>(plan, launch, st, max_blocks);
  }
  if (head_dim == 128) {
    if (kpg == 8) return persist_setup<8, 128, false>(plan, launch, st, max_blocks);
    if (kpg == 4) return persist_setup<4, 128, false>(plan, launch, st, max_blocks);
    return persist_setup<16, 128, false>(plan, launch, st, max_blocks);
  }
  if (kpg == 8) return persist_setup<8, 64, false>(plan, launch, st, max_blocks);
  if (kpg == 4) return persist_setup<4, 64, false>(plan, launch, st, max_blocks);
  return persist_setup<16, 64, false>(plan, launch, st, max_blocks);
}

int persist_plan(const PdPhase* ph, int n, int head_dim, int group_q, int page_size, int tp_size, PdPlan* plan) {
  auto round = [](size_t v) { return (v + 127) / 128 * 128; };
  if (!(head_dim == 64 || head_dim == 128) || group_q < 1 || group_q > PD_MAXG || page_size != PD_PAGE)
    return N730_UNSUPPORTED;
  int dev = 0, sms = 0, coop = 0, maxb = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  N730_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  if (!coop) return N730_UNSUPPORTED;
  int kpg = 0, kmax = 0, gmax = 0, ffn_floats = 0;
  bool mixed = false;
  for (int i = 0; i < n; ++i) {
    if (ph[i].kind != PD_GEMV && ph[i].kind != PD_FFN) continue;
    if (ph[i].prec == 8 || ph[i].prec == 16) {  // INT8 / FP16 tiles: GEMV phases, 128-column units
      if (ph[i].kind != PD_GEMV || ph[i].cols % PD_TILE_K || ph[i].G != ph[i].cols / PD_TILE_K) return N730_UNSUPPORTED;
      mixed = true;
    } else if (ph[i].prec != 0 && ph[i].prec != 4) {
      return N730_UNSUPPORTED;
    }
    const int k = ph[i].cols / ph[i].G / 16;
    if (ph[i].cols % 64 || (ph[i].norm_w && ph[i].cols > PD_KNORM) || (kpg && k != kpg) ||
        !(k == 4 || k == 8 || k == 16))
      return N730_UNSUPPORTED;
    if (ph[i].epi == PD_EPI_SWIGLU && ph[i].rows % 2) return N730_UNSUPPORTED;
    if (ph[i].xsum && (!ph[i].norm_w || ph[i].kind != PD_GEMV)) return N730_UNSUPPORTED;
    int tiles_per_cta = ((ph[i].rows + 15) / 16 + sms - 1) / sms;
    if ((int64_t)((ph[i].rows + 15) / 16) * ph[i].G * std::max(sms, PD_WARPS) >= (1ll << 31)) return N730_UNSUPPORTED;
    if (ph[i].kind == PD_FFN) {
      // gate|up rows interleave the down_proj input channels; whole down groups per CTA
      const int nj = (ph[i].G2 + sms - 1) / sms;
      if (ph[i].epi != PD_EPI_SWIGLU || ph[i].rows != 2 * ph[i].cols2 || ph[i].cols2 != ph[i].G2 * 16 * k ||
          nj > PD_FFN_MAXG || nj > pd_gpc(k) || nj * 16 * k > ph[i].cols || !ph[i].acc)
        return N730_UNSUPPORTED;
      tiles_per_cta = nj * 2 * k;
      kmax = std::max(kmax, nj * 16 * k);
      gmax = std::max(gmax, nj);
      ffn_floats = std::max(ffn_floats, nj * 16 * k);
    }
    if ((ph[i].epi == PD_EPI_RESID || ph[i].bias) && tiles_per_cta * 16 > PD_ADDMAX) return N730_UNSUPPORTED;
    kpg = k;
    kmax = std::max(kmax, ph[i].cols);
    gmax = std::max(gmax, ph[i].G);
  }
  if (!kpg) return N730_UNSUPPORTED;
  PdArgs& a = plan->a;
  a.kpg = kpg;
  a.tp_size = tp_size;
  a.mixed = mixed;
  const int gb = kpg * 128 + 64;
  a.ring_stride = (int)round((size_t)pd_gpc(kpg) * gb);
  if (mixed && a.ring_stride < PD_UNIT16) return N730_UNSUPPORTED;
  size_t off = round((size_t)(PD_WARPS * PD_RING + 1) * 8);
  a.ring_off = (int)off;
  off += (size_t)PD_WARPS * PD_RING * a.ring_stride;
  a.work_off = (int)round(off);
  const size_t gemv_work = round((size_t)kmax * 2) + (size_t)(gmax + 8) * 4;
  const size_t attn_work = ((size_t)PD_MAXG * head_dim + PD_MAXG * PD_PAGE + PD_MAXG * 4 + 8 * PD_MAXSPLIT +
                            (size_t)PD_MAXG * head_dim + PD_MAXSPLIT) * 4;
  off = a.work_off + round(std::max(gemv_work, attn_work));
  a.kv_off = (int)off;
  off += round((size_t)2 * PD_PAGE * head_dim * 2);
  a.add_off = (int)off;
  off += round((size_t)PD_ADDMAX * 4);
  a.wpart_off = (int)off;
  off += round((size_t)PD_WARPS * 2 * 16 * 4);
  a.misc_off = (int)off;
  off += 96 * 4;
  a.ffn_off = (int)round(off);
  off = a.ffn_off + (size_t)ffn_floats * 4;
  a.tab_off = (int)round(off);
  if (round(a.tab_off + (size_t)n * sizeof(PdPhase)) <= 227 * 1024) {
    off = a.tab_off + (size_t)n * sizeof(PdPhase);
  } else {  // the phase table stays in global memory
    off = a.tab_off;
    a.tab_off = -1;
  }
  plan->smem = round(off);
  if (plan->smem > 227 * 1024) return N730_UNSUPPORTED;
  a.d.head_dim = head_dim;
  if (int rc = persist_dispatch(*plan, head_dim, false, nullptr, &maxb)) return rc;
  if (maxb < 1) return N730_UNSUPPORTED;
  plan->grid = sms;
  return N730_OK;
}

// ---- INT8 / FP16 weights as persistent tiles (layout in decode_persist.h) ----
__device__ __forceinline__ float2 pd_sz_rowmajor(const QWeight& w, int r, int c) {
  const uint8_t* row = reinterpret_cast<const uint8_t*>(w.sz) + (int64_t)r * w.sz_pitch;
  if (w.sz_mode == 0) return __half22float2(reinterpret_cast<const __half2*>(row)[c / w.group]);
  return *reinterpret_cast<const float2*>(row);
}

// one thread per output element of a unit (codes; then the 32 scale/zero floats for INT8)
__global__ void pd_tile_kernel(const QWeight w, uint8_t* out, int G) {
  const int per = w.bits == 8 ? 16 * PD_TILE_K + 32 : 16 * PD_TILE_K;
  const int64_t n = (int64_t)((w.rows + 15) / 16) * G * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t unit = i / per;
    const int e = (int)(i - unit * per);
    const int t = (int)(unit / G), j = (int)(unit - (int64_t)t * G);
    if (w.bits == 8) {
      uint8_t* ub = out + unit * PD_UNIT8;
      if (e >= 16 * PD_TILE_K) {  // {scale_g, zero_g, scale_g+8, zero_g+8}, g = 0..7
        const int f = e - 16 * PD_TILE_K, g = f >> 2, k = f & 3;
        const int r = t * 16 + g + 8 * (k >> 1);
        float v = 0.f;
        if (r < w.rows) {
          const float2 sz = pd_sz_rowmajor(w, r, j * PD_TILE_K);
          v = (k & 1) ? sz.y : sz.x;
        }
        reinterpret_cast<float*>(ub + 16 * PD_TILE_K)[f] = v;
        continue;
      }
      const int s2 = e >> 9, rem = e & 511, lane = rem >> 4, b = rem & 15;
      const int s = s2 * 2 + (b >> 3), kh = (b >> 2) & 1, h = (b >> 1) & 1, el = b & 1;
      const int r = t * 16 + (lane >> 2) + 8 * h;
      const int c = j * PD_TILE_K + s * 16 + 2 * (lane & 3) + el + 8 * kh;
      ub[e] = r < w.rows ? w.codes[(int64_t)r * w.row_bytes + c] : (uint8_t)0;
    } else {
      __half* ub = reinterpret_cast<__half*>(out + unit * PD_UNIT16);
      const int s = e >> 8, rem = e & 255, lane = rem >> 3, q = rem & 7;
      const int reg = q >> 1, el = q & 1, h = reg & 1, kh = reg >> 1;
      const int r = t * 16 + (lane >> 2) + 8 * h;
      const int c = j * PD_TILE_K + s * 16 + 2 * (lane & 3) + el + 8 * kh;
      ub[e] = r < w.rows ? reinterpret_cast<const __half*>(w.codes + (int64_t)r * w.row_bytes)[c] : __float2half(0.f);
    }
  }
}

int64_t pd_tile_bytes(int bits, int rows, int cols) {
  const int64_t units = (int64_t)((rows + 15) / 16) * (cols / PD_TILE_K);
  return units * (bits == 8 ? PD_UNIT8 : PD_UNIT16);
}

int pd_tile_launch(const QWeight& w, uint8_t* out, cudaStream_t st) {
  N730_REQUIRE((w.bits == 8 || w.bits == 16) && w.layout == 0 && w.cols % PD_TILE_K == 0, N730_UNSUPPORTED,
               "persistent tiles: %d-bit weight, layout %d, %d columns", w.bits, w.layout, w.cols);
  N730_REQUIRE(w.bits == 16 || w.sz_mode == 1 || w.group % PD_TILE_K == 0, N730_UNSUPPORTED,
               "persistent tiles: INT8 group %d", w.group);
  const int G = w.cols / PD_TILE_K;
  const int64_t n = (int64_t)((w.rows + 15) / 16) * G * (w.bits == 8 ? 16 * PD_TILE_K + 32 : 16 * PD_TILE_K);
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 65536);
  pd_tile_kernel<<<blocks, 256, 0, st>>>(w, out, G);
  N730_CUDA(cudaGetLastError());
  return N730_OK;
}

// down_proj units in group-major order for the fused FFN: unit (t, g) of the
// fragment tiles (byte (t * G + g) * gb) moves to byte (g * T + t) * gb, so the
// row tiles of one group (one CTA's slice) are contiguous and a chunk of them
// is one bulk copy.
__global__ void pd_group_major_kernel(const uint4* src, uint4* dst, int T, int G, int words) {
  const int64_t n = (int64_t)T * G * words;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t unit = i / words;
    const int w = (int)(i - unit * words);
    const int t = (int)(unit / G), g = (int)(unit - (int64_t)t * G);
    dst[((int64_t)g * T + t) * words + w] = src[i];
  }
}

int pd_group_major_launch(const uint8_t* tiles, int rows, int n_groups, int group, uint8_t* out, cudaStream_t st) {
  const int gb = (group / 16) * 128 + 64;
  N730_REQUIRE(gb % 16 == 0 && ((uintptr_t)tiles & 15) == 0 && ((uintptr_t)out & 15) == 0, N730_BAD_ARG,
               "group-major copy: alignment");
  const int T = (rows + 15) / 16;
  const int64_t n = (int64_t)T * n_groups * (gb / 16);
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 65536);
  pd_group_major_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const uint4*>(tiles), reinterpret_cast<uint4*>(out),
                                                T, n_groups, gb / 16);
  N730_CUDA(cudaGetLastError());
  return N730_OK;
}

int persist_grid(int* grid) {
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_CUDA(cudaDeviceGetAttribute(grid, cudaDevAttrMultiProcessorCount, dev));
  return N730_OK;
}

int persist_launch(const PdPlan& plan, cudaStream_t st) {
  return persist_dispatch(plan, plan.a.d.head_dim, true, st, nullptr);
}

}  // namespace n730
