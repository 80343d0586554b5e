// Persistent single-launch decode step (batch 1, INT4 fragment-tiled weights).
#pragma once
#include <cstdint>

#include "attention.h"

namespace n730 {

enum : int { PD_GEMV = 0, PD_ATTN = 1, PD_FFN = 2 };
enum : int { PD_EPI_STORE = 0, PD_EPI_RESID = 1, PD_EPI_SWIGLU = 2, PD_EPI_XPUSH = 3 };
constexpr int PD_MAX_RANKS = 8;

// One op of the step.  GEMV: y (+)= W x with W in fragment tiles (`blob`,
// rows x cols, G groups per row), optional RMSNorm of x (`norm_w`) and bias;
// epilogue store, residual add in place, or SwiGLU of interleaved gate/up rows
// (y[r/2] = silu(gate) * up).  ATTN: RoPE + GQA attention of the step's qkv
// against layer `kv`.
// FFN: the MLP without a grid barrier between its two GEMVs.  CTA c owns whole
// quantisation groups [j0, j1) of down_proj's input (the FFN channels); it
// computes the gate|up rows of exactly those channels (`blob`, interleaved,
// SwiGLU into shared memory) and then down_proj's partial sums over them for
// every output row (`blob2`: rows2 x cols2, G2 groups, units in group-major
// order so a CTA's groups are contiguous: pd_group_major_launch), added into `acc` as
// 32.32 fixed-point integers (integer addition is associative, so the sum is
// the same whatever order the CTAs arrive in).  The residual stream is then
// h + acc: a later GEMV with a non-null `acc` reads x + acc (norm phases) or,
// with the residual epilogue, folds acc into y and clears it.
// Tensor parallel (several ranks, one launch per rank): a row-split GEMV
// (o_proj / down_proj over this rank's K columns) ends with PD_EPI_XPUSH: each
// row's partial sum is stored into slot [xpar][rank] of EVERY rank's exchange
// area (peer memory).  The barrier before the next GEMV is then cross-GPU
// (`xbar`), and its prologue (`xsum`) reads x = h + sum over ranks of slot
// [xpar][r] in rank order (identical on every rank), the CTA owning a row
// range also writing the new residual to `h_out` (the other residual buffer).
struct __align__(16) PdPhase {
  int8_t kind, epi;
  int8_t xpar, xsum;        // tensor parallel: exchange slot parity; x = h + sum of the ranks' slots
  int16_t xbar;             // tensor parallel: the barrier before this phase is cross-GPU barrier xbar (0: local)
  int8_t prec;              // weight tiles: 4 INT4 fragment tiles (0 reads as 4), 8 INT8, 16 FP16 (PdTile*)
  int8_t pad_;
  const uint8_t* blob;
  int rows, cols, G;
  int rows2;                // FFN: down_proj rows
  const float* x;
  const float* norm_w;
  const float* bias;
  float* y;
  KVLayer kv;
  const uint8_t* blob2;     // FFN: down_proj, group-major fragment tiles
  int cols2, G2;
  unsigned long long* acc;  // FFN: down_proj sums (fixed point, 2^-32); GEMV: pending residual
  float* h_out;             // tensor parallel: residual stream after this exchange
};

static_assert(sizeof(PdPhase) % 16 == 0, "phase table rows are copied as words");
static_assert(sizeof(PdPhase) == 112, "an 80-layer phase table (fused FFN) must fit in shared memory");

// Weight tiles of the persistent kernel for INT8 (per-tensor, per-channel or
// grouped scale/zero) and FP16 weights, one unit per 16 rows x 128 columns,
// units [row tile][column block] like the INT4 fragment tiles:
//   INT8: 2048 B codes, [k-step pair][lane][16 B]: per k-step 8 B = the A
//         fragment of mma.m16n8k16 (rows g / g+8, columns 2tq.. / 2tq+8..) as
//         bytes {a0.0, a0.1, a1.0, a1.1, a2.0, a2.1, a3.0, a3.1}; then 128 B
//         {scale_g, zero_g, scale_g+8, zero_g+8} fp32 per g = 0..7.
//   FP16: 4096 B, [k-step][lane][16 B]: the four A fragment registers.
constexpr int PD_TILE_K = 128;
constexpr int PD_UNIT8 = 16 * PD_TILE_K + 128;
constexpr int PD_UNIT16 = 16 * PD_TILE_K * 2;
// Bytes of the tiles of an INT8 / FP16 weight (rows x cols, cols % 128 == 0).
int64_t pd_tile_bytes(int bits, int rows, int cols);
// Write weight `w` (INT8 row-major with scale/zero, or FP16) as persistent tiles into `out`.
struct QWeight;
int pd_tile_launch(const QWeight& w, uint8_t* out, cudaStream_t st);
// Copy of INT4 fragment tiles (rows x n_groups groups of `group`) with units in
// group-major order [group][row tile]: the fused FFN's down_proj (`blob2`).
int pd_group_major_launch(const uint8_t* tiles, int rows, int n_groups, int group, uint8_t* out, cudaStream_t st);

struct PdArgs {
  const PdPhase* phases;
  int n_phases;
  int kpg;                  // k-steps per group (group / 16), the same for every GEMV
  float eps;
  // attention (batch 1)
  const float* qkv;         // [n_heads + 2 n_kv][head_dim]: q | k | v of the new token
  float* attn_out;          // [n_heads * head_dim]
  const float* cos_t;
  const float* sin_t;
  const int* seq_lens;      // [0]: tokens already cached
  const int* block_table;   // sequence 0's page row
  AttnDims d;
  int max_split;            // context splits per KV head (n_kv * max_split <= grid)
  float* attn_part;         // [n_kv * max_split][G_q][head_dim + 2]
  int* attn_cnt;            // [n_kv]            zero between launches
  int* sync;                // [0] arrivals, [1] exits, [2] abort   zero between launches
  int* err;                 // device error word (DEV_ERR_TIMEOUT on a wait that ran out)
  unsigned long long* acc;  // FFN accumulator [acc_n], cleared by the last CTA out
  int acc_n;
  // shared-memory layout (bytes); tab_off < 0: the phase table is read from global memory
  int ring_off, ring_stride, work_off, kv_off, add_off, wpart_off, misc_off, ffn_off, tab_off;
  // tensor parallel (tp_size > 1): exchange areas [2 parity][tp_size][xcap] floats and
  // cross-barrier counters of every rank (own at tp_rank), mapped into this process
  int tp_rank, tp_size;
  int64_t xcap;
  float* xrecv[PD_MAX_RANKS];
  int* xcnt[PD_MAX_RANKS];
  float* xrecv_local;       // xrecv[tp_rank]
  int* xcnt_local;          // xcnt[tp_rank]
  int* xepoch;              // launches completed on this rank (the same count on every rank)
  int n_xbar;               // cross barriers per launch
  int mixed;                // some phases stream INT8 / FP16 tiles (set by persist_plan)
  // per-phase timing (null: off): [PD_TRACE_ROWS * n_phases + 1][grid] %globaltimer ns; for
  // phase p, row 6p: the CTA's arrival at the barrier before it (p = 0: launch start), 6p+1: its
  // departure from it (the start of phase p), 6p+2 and 6p+3: marks inside the phase (GEMV:
  // prologue done; FFN: prologue done, gate|up done; attention: split partial written, head's
  // splits all published; 0 where a CTA has none), 6p+4 and 6p+5: ns its warps spent waiting
  // for weight chunks, summed over the warps (GEMV or gate|up; down_proj); the last row: the
  // end of its last phase
  unsigned long long* trace;
};
constexpr int PD_TRACE_ROWS = 6;

struct PdPlan {
  PdArgs a{};
  int grid = 0;
  size_t smem = 0;
};

// Shared-memory layout and grid for `phases` (host copy); N730_UNSUPPORTED if
// the step cannot run persistently (the caller then uses the per-op kernels).
// The KV cache must use pages of PD_PAGE positions.  FFN phases need at most
// PD_FFN_MAXG down groups per CTA.
constexpr int PD_PAGE = 64;
constexpr int PD_FFN_MAXG = 4;
// CTAs of the persistent launch on the current device (one per SM)
int persist_grid(int* grid);
int persist_plan(const PdPhase* host_phases, int n_phases, int head_dim, int group_q, int page_size, int tp_size,
                 PdPlan* plan);
int persist_launch(const PdPlan& plan, cudaStream_t st);

}  // namespace n730
