// Persistent single-launch decode step (batch 1, INT4 fragment-tiled weights).
#pragma once
#include "attention.h"

namespace n730 {

enum : int { PD_GEMV = 0, PD_ATTN = 1, PD_FFN = 2 };
enum : int { PD_EPI_STORE = 0, PD_EPI_RESID = 1, PD_EPI_SWIGLU = 2 };

// One op of the step.  GEMV: y (+)= W x with W in fragment tiles (`blob`,
// rows x cols, G groups per row), optional RMSNorm of x (`norm_w`) and bias;
// epilogue store, residual add in place, or SwiGLU of interleaved gate/up rows
// (y[r/2] = silu(gate) * up).  ATTN: RoPE + GQA attention of the step's qkv
// against layer `kv`.
// FFN: the MLP without a grid barrier between its two GEMVs.  CTA c owns whole
// quantisation groups [j0, j1) of down_proj's input (the FFN channels); it
// computes the gate|up rows of exactly those channels (`blob`, interleaved,
// SwiGLU into shared memory) and then down_proj's partial sums over them for
// every output row (`blob2`: rows2 x cols2, G2 groups), added into `acc` as
// 32.32 fixed-point integers (integer addition is associative, so the sum is
// the same whatever order the CTAs arrive in).  The residual stream is then
// h + acc: a later GEMV with a non-null `acc` reads x + acc (norm phases) or,
// with the residual epilogue, folds acc into y and clears it.
struct __align__(16) PdPhase {
  int kind, epi;
  const uint8_t* blob;
  int rows, cols, G;
  const float* x;
  const float* norm_w;
  const float* bias;
  float* y;
  KVLayer kv;
  const uint8_t* blob2;     // FFN: down_proj
  int rows2, cols2, G2;
  unsigned long long* acc;  // FFN: down_proj sums (fixed point, 2^-32); GEMV: pending residual
};

static_assert(sizeof(PdPhase) % 16 == 0, "phase table rows are copied as words");

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
  // shared-memory layout (bytes)
  int ring_off, ring_stride, work_off, kv_off, add_off, wpart_off, misc_off, ffn_off, tab_off;
};

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
int persist_plan(const PdPhase* host_phases, int n_phases, int head_dim, int group_q, int page_size, PdPlan* plan);
int persist_launch(const PdPlan& plan, cudaStream_t st);

}  // namespace n730
