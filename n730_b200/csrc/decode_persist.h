// Persistent single-launch decode step (batch 1, INT4 fragment-tiled weights).
#pragma once
#include "attention.h"

namespace n730 {

enum : int { PD_GEMV = 0, PD_ATTN = 1 };
enum : int { PD_EPI_STORE = 0, PD_EPI_RESID = 1, PD_EPI_SWIGLU = 2 };

// One op of the step.  GEMV: y (+)= W x with W in fragment tiles (`blob`,
// rows x cols, G groups per row), optional RMSNorm of x (`norm_w`) and bias;
// epilogue store, residual add in place, or SwiGLU of interleaved gate/up rows
// (y[r/2] = silu(gate) * up).  ATTN: RoPE + GQA attention of the step's qkv
// against layer `kv`.
struct PdPhase {
  int kind, epi;
  const uint8_t* blob;
  int rows, cols, G;
  const float* x;
  const float* norm_w;
  const float* bias;
  float* y;
  KVLayer kv;
};

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
  // shared-memory layout (bytes)
  int ring_off, ring_stride, work_off, kv_off, add_off, wpart_off, misc_off;
};

struct PdPlan {
  PdArgs a{};
  int grid = 0;
  size_t smem = 0;
};

// Shared-memory layout and grid for `phases` (host copy); N730_UNSUPPORTED if
// the step cannot run persistently (the caller then uses the per-op kernels).
// The KV cache must use pages of PD_PAGE positions.
constexpr int PD_PAGE = 64;
int persist_plan(const PdPhase* host_phases, int n_phases, int head_dim, int group_q, int page_size, PdPlan* plan);
int persist_launch(const PdPlan& plan, cudaStream_t st);

}  // namespace n730
