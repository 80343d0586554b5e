// Packed weights resident in HBM, and the kernels that consume them.
#pragma once
#include "common.cuh"

namespace n730 {

// Device layout of one linear weight W[rows, cols] (out x in).
//   codes : [rows][row_bytes] packed codes, element 0 of a row in the least
//           significant bits (the .n730 packing), rows padded to 16 bytes.
//           For FP16 weights: [rows][cols] fp16.
//   sz    : sz_mode 0 -> half2 (scale, zero) per (row, group), rows of sz_pitch bytes
//           sz_mode 1 -> float2 (scale, zero) per row, rows of sz_pitch (16) bytes
//           (sz_pitch is a multiple of 16 so a run of rows is one bulk copy)
//           (per-tensor blocks are stored as mode 1 with the tensor's fp32
//           scale and zero point on every row, so dequant stays bit-exact)
// Dequantised value: (float(q) - zero) * scale, fp32, no contraction.
struct QWeight {
  int prec = 0;
  int bits = 0;
  int rows = 0;
  int cols = 0;
  int group = 0;      // elements per group (== cols for sz_mode 1)
  int n_groups = 0;   // groups per row
  int sz_mode = 0;
  int layout = 0;     // 0 row-major padded rows; 1 mma fragment tiles (INT4 grouped)
  int64_t row_bytes = 0;
  int64_t sz_pitch = 0;
  uint8_t* codes = nullptr;
  void* sz = nullptr;
  bool owns = true;
  int device = 0;
};

// rows per sum of squares that a split-K fold hands to the next RMSNorm (GemvArgs::ss_out / ss_in)
constexpr int TC_SS_ROWS = 256;

struct GemvArgs {
  const QWeight* w;
  const float* x;        // [batch][ldx] fp32 activations
  int ldx;
  int batch;
  float* y;              // [batch][ldy]
  int ldy;
  const float* bias;     // [rows] or null
  const float* residual; // [batch][ldr] or null; y = residual + W x (+ bias); may alias y
  int ldr;
  const float* norm_w;   // [cols] RMSNorm weight applied to x first, or null
  float eps;
  int swiglu;            // rows interleaved gate/up: y[b][r/2] = silu(g)*u
  int pdl;               // launched with programmatic dependent launch
  float* split_ws;       // tensor-core GEMV: workspace for split-K partial sums (null: one K pass per
  int64_t split_ws_floats;  //   batch chunk that fits shared memory)
  // tcgen05 GEMM only (null elsewhere):
  float* ss_out;         // with split K (gemm_tc_folds): the fold also writes the sums of squares of y,
                         //   [batch][ceil(rows / TC_SS_ROWS)], one per 256-row slice of each token
  const float* ss_in;    // with norm_w: 1/rms of x from such sums ([batch][ceil(cols / TC_SS_ROWS)])
                         //   instead of a pass over x of its own
};

int gemv_launch(const GemvArgs& a, cudaStream_t stream);
int gemv_mma_launch(const GemvArgs& a, cudaStream_t stream);
// tcgen05 GEMM for many tokens (gemm_tc.cu); inv_ws: batch floats of workspace when norm_w is set
bool gemm_tc_supported(const QWeight& w, int tokens);
int gemm_tc_prepare();
// workspaces for calls of up to `tokens` tokens, `cols` columns and `rows` rows (before any capture)
int gemm_tc_reserve(int tokens, int cols, int rows, cudaStream_t stream);
int gemm_tc_tile(int row_tiles, int tokens);
// true when a call of `tokens` tokens splits K and folds the parts (the fold can write ss_out)
bool gemm_tc_folds(const QWeight& w, int tokens, bool swiglu);
int gemm_tc_ctas(int rows, int cols, int tokens, bool swiglu);
// from this many rows of x on, model linears take the tcgen05 GEMM (each weight dequantised
// once for up to 256 rows); below it the GEMV (weights streamed once per 16 rows), except
// where the model's rule prefers the GEMM (wide linears at 17-127 rows)
constexpr int GEMM_TC_MIN_TOKENS = 128;
int gemm_tc_launch(const GemvArgs& a, float* inv_ws, cudaStream_t stream);
int qweight_to_mma_layout(QWeight& w, cudaStream_t stream);
int* gemv_err_word();
int gemv_check_error(bool reset);
int gemv_prepare();  // allocate device state before any graph capture  // N730_TIMEOUT if a device wait ran out
int dequant_launch(const QWeight& w, float* out, int64_t ld_out, int row0, int nrows,
                   cudaStream_t stream);
int repack_rows_launch(const uint8_t* src, int bits, int rows, int cols, uint8_t* dst,
                       int64_t row_bytes, cudaStream_t stream);
int fill_f2_launch(void* out, int64_t pitch, int n, float a, float b, cudaStream_t stream);
int64_t sz_pitch_for(int sz_mode, int n_groups);
int embed_launch(const QWeight& w, const int32_t* tokens, int n, float* out, cudaStream_t stream);

}  // namespace n730
