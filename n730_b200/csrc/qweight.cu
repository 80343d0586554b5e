// Packed-weight registration, bit-exact dequant, embedding gather, GPU
// group-wise quantiser, and their C entry points.
#include <algorithm>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "qweight.h"

namespace n730 {

static thread_local std::string g_err;
void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}
const char* last_error() { return g_err.c_str(); }

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t code_at(const uint8_t* row, int bits, int c) {
  const int bit = c * bits;
  return (row[bit >> 3] >> (bit & 7)) & ((1u << bits) - 1u);
}

// (float(q) - zero) * scale with the subtraction and multiplication rounded
// separately (no FMA contraction): n730core.cpp:65,80-82,98-101.
__device__ __forceinline__ float dq(uint32_t q, float s, float z) {
  return __fmul_rn(__fsub_rn((float)q, z), s);
}

__device__ __forceinline__ float2 load_sz(const QWeight& w, int r, int c) {
  if (w.layout == 1) {  // fragment tiles: per (tile, group) codes then {s_g, s_g8, z_g, z_g8} x 8
    const int t = r >> 4, rr = r & 15, g = rr & 7, kpg = w.group >> 4;
    const uint8_t* grp = w.codes + ((int64_t)t * w.n_groups + c / w.group) * ((int64_t)kpg * 128 + 64);
    const uint2 v = reinterpret_cast<const uint2*>(grp + kpg * 128)[g];
    const __half2 sc = *reinterpret_cast<const __half2*>(&v.x), zp = *reinterpret_cast<const __half2*>(&v.y);
    return rr < 8 ? make_float2(__low2float(sc), __low2float(zp)) : make_float2(__high2float(sc), __high2float(zp));
  }
  const uint8_t* row = reinterpret_cast<const uint8_t*>(w.sz) + (int64_t)r * w.sz_pitch;
  if (w.sz_mode == 0) return __half22float2(reinterpret_cast<const __half2*>(row)[c / w.group]);
  return *reinterpret_cast<const float2*>(row);
}

// code of element (r, c); layout 1 inverts the fragment packing of gemv_mma.cu
__device__ __forceinline__ uint32_t code_rc(const QWeight& w, int r, int c) {
  if (w.layout == 1) {
    const int t = r >> 4, rr = r & 15, kpg = w.group >> 4;
    const int s = (c % w.group) >> 4, kc = c & 15;  // k-step within the group, column within the k-step
    const int lane = (rr & 7) * 4 + ((kc & 7) >> 1);
    const int nib = (rr >> 3) + 2 * (kc >> 3) + 4 * (kc & 1);
    const uint8_t* grp = w.codes + ((int64_t)t * w.n_groups + c / w.group) * ((int64_t)kpg * 128 + 64);
    const uint32_t word = reinterpret_cast<const uint32_t*>(grp)[((s >> 2) * 32 + lane) * 4 + (s & 3)];
    return (word >> (4 * nib)) & 15u;
  }
  return code_at(w.codes + (int64_t)r * w.row_bytes, w.bits, c);
}

__global__ void dequant_kernel(const QWeight w, float* out, int64_t ld, int row0, int nrows) {
  const int64_t n = (int64_t)nrows * w.cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = row0 + (int)(i / w.cols), c = (int)(i % w.cols);
    float v;
    if (w.bits == 16) {
      v = __half2float(reinterpret_cast<const __half*>(w.codes + (int64_t)r * w.row_bytes)[c]);
    } else {
      const float2 sz = load_sz(w, r, c);
      v = dq(code_rc(w, r, c), sz.x, sz.y);
    }
    out[(int64_t)(r - row0) * ld + c] = v;
  }
}

__global__ void embed_kernel(const QWeight w, const int32_t* tokens, int n, float* out) {
  const int t = blockIdx.y;
  if (t >= n) return;
  const int r = tokens[t];
  if (r < 0 || r >= w.rows) {  // out-of-range id: emit zeros (host validates ids)
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < w.cols; c += gridDim.x * blockDim.x)
      out[(int64_t)t * w.cols + c] = 0.f;
    return;
  }
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < w.cols; c += gridDim.x * blockDim.x) {
    float v;
    if (w.bits == 16) v = __half2float(reinterpret_cast<const __half*>(w.codes + (int64_t)r * w.row_bytes)[c]);
    else { const float2 sz = load_sz(w, r, c); v = dq(code_rc(w, r, c), sz.x, sz.y); }
    out[(int64_t)t * w.cols + c] = v;
  }
}

// flat-packed codes (file layout) -> rows padded to row_bytes
__global__ void repack_rows_kernel(const uint8_t* src, int bits, int rows, int cols,
                                   uint8_t* dst, int64_t row_bytes) {
  const int64_t n = (int64_t)rows * row_bytes;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / row_bytes);
    const int64_t j = i % row_bytes;
    uint8_t out = 0;
    if (bits >= 8) {
      const int64_t rb = (int64_t)cols * (bits / 8);
      if (j < rb) out = src[(int64_t)r * rb + j];
    } else {
      const int per = 8 / bits;
      for (int k = 0; k < per; ++k) {
        const int64_t c = j * per + k;
        if (c < cols) {
          const int64_t e = (int64_t)r * cols + c;
          const int64_t bit = e * bits;
          const uint32_t q = (src[bit >> 3] >> (bit & 7)) & ((1u << bits) - 1u);
          out |= (uint8_t)(q << (k * bits));
        }
      }
    }
    dst[i] = out;
  }
}

// s16/z16 [rows][G] -> half2 rows of `pitch` bytes (padding zeroed)
__global__ void interleave_sz_kernel(const __half* s, const __half* z, int rows, int G, int64_t pitch,
                                     uint8_t* out) {
  const int64_t per = pitch / 4, n = (int64_t)rows * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per, g = i % per;
    __half2 v = __halves2half2(__float2half(0.f), __float2half(0.f));
    if (g < G) v = __halves2half2(s[r * G + g], z[r * G + g]);
    reinterpret_cast<__half2*>(out)[i] = v;
  }
}

__global__ void fill_f2_kernel(uint8_t* out, int64_t pitch, int n, float a, float b) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    *reinterpret_cast<float4*>(out + (int64_t)i * pitch) = make_float4(a, b, 0.f, 0.f);
}

// Group-wise quantiser; the arithmetic restates the converter's per-group rule:
// INT4/INT2: scale = fp16((max-min)/qmax) from float64, zp = clip(rint(-min/s), 0, qmax)
// in float64, q = clip(rint(w/s) + zp, 0, qmax) with an fp32 division.
// INT8: s = fp16(absmax/127), q = clip(rint(w/s), -127, 127) + 128, zero 128.
// Degenerate groups (range < 1e-9 or fp16 scale == 0): codes 0, scale 1, zero 0.
// One warp per group (group <= 32 * 64).
__global__ void quantize_grouped_kernel(const float* w, int rows, int cols, int bits, int group,
                                        uint8_t* codes, __half* s16, __half* z16, int* overflow) {
  const int G = cols / group;
  const int64_t ngroups = (int64_t)rows * G;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t gi = gw; gi < ngroups; gi += nw) {
    const int r = (int)(gi / G), g = (int)(gi % G);
    const float* src = w + (int64_t)r * cols + (int64_t)g * group;
    float mn = INFINITY, mx = -INFINITY, am = 0.f;
    for (int i = lane; i < group; i += 32) {
      const float v = src[i];
      mn = fminf(mn, v); mx = fmaxf(mx, v); am = fmaxf(am, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    }
    const int qmax = (1 << bits) - 1;
    bool degen;
    double scale64;
    if (bits == 8) { degen = (double)am < 1e-9; scale64 = (double)am / 127.0; }
    else { degen = fabs((double)mx - (double)mn) < 1e-9; scale64 = ((double)mx - (double)mn) / (double)qmax; }
    __half sh = __double2half(scale64);
    float s = __half2float(sh);
    if (!degen && isinf(s) && lane == 0) atomicExch(overflow, 1);
    if (s == 0.f) degen = true;
    float zp;
    if (degen) { s = 1.f; sh = __float2half(1.f); zp = 0.f; }
    else if (bits == 8) zp = 128.f;
    else zp = (float)fmin(fmax(rint(-(double)mn / (double)s), 0.0), (double)qmax);
    if (lane == 0) { s16[gi] = sh; z16[gi] = __float2half(zp); }
    // codes: each lane builds whole bytes
    const int per = 8 / bits;
    const int nbytes = group / per;
    uint8_t* dst = codes + ((int64_t)r * cols + (int64_t)g * group) * bits / 8;
    for (int j = lane; j < nbytes; j += 32) {
      uint32_t byte = 0;
      for (int k = 0; k < per; ++k) {
        const float v = src[j * per + k];
        uint32_t q;
        if (degen) q = 0;
        else if (bits == 8) q = (uint32_t)(fminf(fmaxf(rintf(__fdiv_rn(v, s)), -127.f), 127.f) + 128.f);
        else q = (uint32_t)fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(v, s)), zp), 0.f), (float)qmax);
        byte |= q << (k * bits);
      }
      dst[j] = (uint8_t)byte;
    }
  }
}

static int grid_for(int64_t n, int block = 256) {
  int64_t g = (n + block - 1) / block;
  const int cap = num_sms() * 16;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

int dequant_launch(const QWeight& w, float* out, int64_t ld, int row0, int nrows, cudaStream_t st) {
  if (nrows <= 0) return N730_OK;
  dequant_kernel<<<grid_for((int64_t)nrows * w.cols), 256, 0, st>>>(w, out, ld, row0, nrows);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

int repack_rows_launch(const uint8_t* src, int bits, int rows, int cols, uint8_t* dst, int64_t row_bytes,
                       cudaStream_t st) {
  repack_rows_kernel<<<grid_for(rows * row_bytes), 256, 0, st>>>(src, bits, rows, cols, dst, row_bytes);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

int64_t sz_pitch_for(int sz_mode, int n_groups) {
  return sz_mode == 0 ? ((int64_t)n_groups * 4 + 15) / 16 * 16 : 16;
}

int fill_f2_launch(void* out, int64_t pitch, int n, float a, float b, cudaStream_t st) {
  fill_f2_kernel<<<grid_for(n), 256, 0, st>>>((uint8_t*)out, pitch, n, a, b);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

int embed_launch(const QWeight& w, const int32_t* tokens, int n, float* out, cudaStream_t st) {
  if (n <= 0) return N730_OK;
  dim3 grid((w.cols + 255) / 256, n);
  embed_kernel<<<grid, 256, 0, st>>>(w, tokens, n, out);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

// ---------------------------------------------------------------------------
// creation
// ---------------------------------------------------------------------------
static int64_t padded_row_bytes(int bits, int cols) {
  const int64_t rb = ((int64_t)cols * bits + 7) / 8;
  return (rb + 15) / 16 * 16;
}

int qweight_create(int prec, int rows, int cols, int group, float scale, float zp,
                   const void* codes, const void* s16, const void* z16, bool src_device,
                   cudaStream_t st, QWeight** out) {
  N730_REQUIRE(out, N730_NULL, "qweight_create: out is null");
  *out = nullptr;
  const int bits = prec_bits(prec);
  N730_REQUIRE(bits, N730_BAD_ARG, "qweight_create: unknown precision id %d", prec);
  N730_REQUIRE(rows > 0 && cols > 0, N730_BAD_ARG, "qweight_create: bad shape %dx%d", rows, cols);
  N730_REQUIRE(codes, N730_NULL, "qweight_create: codes is null");
  const bool grouped = prec_grouped(prec);
  if (grouped) {
    N730_REQUIRE(s16 && z16, N730_NULL, "qweight_create: grouped precision needs scales and zeros");
    const int E = 128 / bits;
    N730_REQUIRE(group > 0 && cols % group == 0 && group % E == 0, N730_BAD_ARG,
                 "qweight_create: group %d invalid for INT%d cols=%d (need cols %% group == 0, "
                 "group %% %d == 0)", group, bits, cols, E);
  }
  QWeight* w = new QWeight();
  w->prec = prec; w->bits = bits; w->rows = rows; w->cols = cols;
  w->row_bytes = padded_row_bytes(bits, cols);
  cudaGetDevice(&w->device);
  const int64_t flat_bytes = ((int64_t)rows * cols * bits + 7) / 8;
  const bool aligned = ((int64_t)cols * bits) % 128 == 0;
  auto fail = [&](int rc) { cudaFree(w->codes); cudaFree(w->sz); delete w; return rc; };
  if (cudaMalloc(&w->codes, rows * w->row_bytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("qweight_create: out of device memory (%lld B)", (long long)(rows * w->row_bytes));
    return fail(N730_OOM);
  }
  const cudaMemcpyKind kind = src_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (aligned) {
    if (int rc = cuda_rc(cudaMemcpyAsync(w->codes, codes, flat_bytes, kind, st), __FILE__, __LINE__)) return fail(rc);
  } else {
    uint8_t* tmp = nullptr;
    const uint8_t* src = (const uint8_t*)codes;
    if (!src_device) {
      if (cudaMalloc(&tmp, flat_bytes) != cudaSuccess) { cudaGetLastError(); return fail(N730_OOM); }
      if (int rc = cuda_rc(cudaMemcpyAsync(tmp, codes, flat_bytes, cudaMemcpyHostToDevice, st), __FILE__, __LINE__)) {
        cudaFree(tmp); return fail(rc);
      }
      src = tmp;
    }
    repack_rows_kernel<<<grid_for(rows * w->row_bytes), 256, 0, st>>>(src, bits, rows, cols, w->codes, w->row_bytes);
    int rc = cuda_rc(cudaGetLastError(), __FILE__, __LINE__);
    if (tmp) { cudaStreamSynchronize(st); cudaFree(tmp); }
    if (rc) return fail(rc);
  }
  if (bits == 16) {
    w->group = cols; w->n_groups = 1; w->sz_mode = 1;
  } else if (grouped) {
    w->group = group; w->n_groups = cols / group; w->sz_mode = 0;
    w->sz_pitch = sz_pitch_for(0, w->n_groups);
    const int64_t n = (int64_t)rows * w->n_groups;
    if (cudaMalloc(&w->sz, rows * w->sz_pitch) != cudaSuccess) { cudaGetLastError(); return fail(N730_OOM); }
    const __half *ds = (const __half*)s16, *dz = (const __half*)z16;
    __half* tmp = nullptr;
    if (!src_device) {
      if (cudaMalloc(&tmp, n * 4) != cudaSuccess) { cudaGetLastError(); return fail(N730_OOM); }
      cudaMemcpyAsync(tmp, s16, n * 2, cudaMemcpyHostToDevice, st);
      cudaMemcpyAsync(tmp + n, z16, n * 2, cudaMemcpyHostToDevice, st);
      ds = tmp; dz = tmp + n;
    }
    interleave_sz_kernel<<<grid_for(rows * w->sz_pitch / 4), 256, 0, st>>>(ds, dz, rows, w->n_groups,
                                                                          w->sz_pitch, (uint8_t*)w->sz);
    int rc = cuda_rc(cudaGetLastError(), __FILE__, __LINE__);
    if (tmp) { cudaStreamSynchronize(st); cudaFree(tmp); }
    if (rc) return fail(rc);
  } else {
    w->group = cols; w->n_groups = 1; w->sz_mode = 1; w->sz_pitch = 16;
    if (cudaMalloc(&w->sz, (size_t)rows * 16) != cudaSuccess) { cudaGetLastError(); return fail(N730_OOM); }
    fill_f2_kernel<<<grid_for(rows), 256, 0, st>>>((uint8_t*)w->sz, 16, rows, scale, zp);
    if (int rc = cuda_rc(cudaGetLastError(), __FILE__, __LINE__)) return fail(rc);
  }
  if (!src_device) {  // host sources may be freed by the caller after return
    if (int rc = cuda_rc(cudaStreamSynchronize(st), __FILE__, __LINE__)) return fail(rc);
  }
  *out = w;
  return N730_OK;
}

void qweight_destroy(QWeight* w) {
  if (!w) return;
  if (w->owns) { cudaFree(w->codes); cudaFree(w->sz); }
  delete w;
}

// Allocate an empty grouped/per-row weight and copy rows of `src` into rows
// dst_row0 + i*stride (builds fused q|k|v and interleaved gate/up weights).
int qweight_alloc_like(const QWeight& proto, int rows, QWeight** out) {
  QWeight* w = new QWeight(proto);
  w->rows = rows; w->codes = nullptr; w->sz = nullptr; w->owns = true;
  cudaGetDevice(&w->device);
  if (cudaMalloc(&w->codes, rows * w->row_bytes) != cudaSuccess) { cudaGetLastError(); delete w; return N730_OOM; }
  size_t szb = w->bits == 16 ? 0 : (size_t)rows * w->sz_pitch;
  if (szb && cudaMalloc(&w->sz, szb) != cudaSuccess) { cudaGetLastError(); cudaFree(w->codes); delete w; return N730_OOM; }
  *out = w;
  return N730_OK;
}

int qweight_copy_rows(QWeight& dst, const QWeight& src, int dst_row0, int stride, cudaStream_t st) {
  N730_REQUIRE(dst.layout == 0 && src.layout == 0, N730_BAD_ARG, "qweight_copy_rows: row layout required");
  N730_REQUIRE(dst.bits == src.bits && dst.row_bytes == src.row_bytes && dst.sz_mode == src.sz_mode &&
               dst.cols == src.cols && (dst.sz_mode != 0 || dst.n_groups == src.n_groups),
               N730_BAD_ARG, "qweight_copy_rows: layouts differ");
  N730_REQUIRE(dst_row0 + (int64_t)(src.rows - 1) * stride < dst.rows, N730_BAD_ARG,
               "qweight_copy_rows: rows out of range");
  N730_CUDA(cudaMemcpy2DAsync(dst.codes + dst_row0 * dst.row_bytes, dst.row_bytes * stride, src.codes,
                              src.row_bytes, src.row_bytes, src.rows, cudaMemcpyDeviceToDevice, st));
  if (src.bits != 16) {
    const size_t e = src.sz_pitch;
    N730_CUDA(cudaMemcpy2DAsync((uint8_t*)dst.sz + dst_row0 * e, e * stride, src.sz, e, e, src.rows,
                                cudaMemcpyDeviceToDevice, st));
  }
  return N730_OK;
}

}  // namespace n730

using namespace n730;

// ---------------------------------------------------------------------------
// C entry points
// ---------------------------------------------------------------------------
N730_API const char* n730_last_error(void) { return last_error(); }

N730_API int n730_qweight_create(int prec_id, int rows, int cols, int group_size, float scale,
                                 float zero_point, const void* codes, const void* scales16,
                                 const void* zeros16, int src_on_device, void* stream, void** out_qw) {
  QWeight* w = nullptr;
  int rc = qweight_create(prec_id, rows, cols, group_size, scale, zero_point, codes, scales16,
                          zeros16, src_on_device != 0, (cudaStream_t)stream, &w);
  if (out_qw) *out_qw = w;
  return rc;
}

N730_API void n730_qweight_destroy(void* qw) { qweight_destroy((QWeight*)qw); }

// info[0..7] = prec, bits, rows, cols, group, n_groups, row_bytes, device bytes
N730_API int n730_qweight_info(void* qw, int64_t* info) {
  if (!qw || !info) return N730_NULL;
  const QWeight* w = (const QWeight*)qw;
  info[0] = w->prec; info[1] = w->bits; info[2] = w->rows; info[3] = w->cols;
  info[4] = w->group; info[5] = w->n_groups; info[6] = w->row_bytes;
  info[7] = w->layout == 1 ? (int64_t)((w->rows + 15) / 16) * w->n_groups * ((int64_t)(w->group / 16) * 128 + 64)
                           : w->rows * w->row_bytes + (w->bits == 16 ? 0 : (int64_t)w->rows * w->sz_pitch);
  return N730_OK;
}

// Convert a weight to a device layout: 0 row-major (any format), 1 tensor-core
// fragment tiles (INT4 group-wise, group % 64 == 0; used by the mma GEMV).
N730_API int n730_qweight_set_layout(void* qw, int layout, void* stream) {
  if (!qw) return N730_NULL;
  QWeight* w = (QWeight*)qw;
  if (layout == w->layout) return N730_OK;
  N730_REQUIRE(layout == 1, N730_UNSUPPORTED, "qweight_set_layout: only row -> fragment tiles is supported");
  return qweight_to_mma_layout(*w, (cudaStream_t)stream);
}

N730_API int n730_dequant_to_f32(void* qw, float* d_out, void* stream) {
  if (!qw || !d_out) return N730_NULL;
  const QWeight* w = (const QWeight*)qw;
  return dequant_launch(*w, d_out, w->cols, 0, w->rows, (cudaStream_t)stream);
}

N730_API int n730_embed(void* qw, const int32_t* d_tokens, int n, float* d_out, void* stream) {
  if (!qw || !d_tokens || !d_out) return N730_NULL;
  return embed_launch(*(const QWeight*)qw, d_tokens, n, d_out, (cudaStream_t)stream);
}

// y[b, :] = (residual[b, :] +) W x[b, :] (+ bias); optional RMSNorm of x and SwiGLU.
N730_API int n730_qlinear(void* qw, const float* d_x, int ldx, int batch, float* d_y, int ldy,
                          const float* d_bias, const float* d_residual, int ldr,
                          const float* d_norm_w, float eps, int swiglu, void* stream) {
  if (!qw) return N730_NULL;
  GemvArgs a = {};
  a.w = (const QWeight*)qw; a.x = d_x; a.ldx = ldx; a.batch = batch; a.y = d_y; a.ldy = ldy;
  a.bias = d_bias; a.residual = d_residual; a.ldr = ldr; a.norm_w = d_norm_w; a.eps = eps;
  // programmatic dependent launch: the GEMV may start while the previous kernel on the stream
  // finishes; it streams only its weights (complete when n730_qweight_create / _set_layout
  // returned) before the dependency wait, and reads x, bias, residual and norm weights after it
  a.swiglu = swiglu; a.pdl = 1;
  return gemv_launch(a, (cudaStream_t)stream);
}

N730_API int n730_qgemm(void* qw, const float* d_x, int ldx, int tokens, float* d_y, int ldy, const float* d_bias,
                        const float* d_residual, int ldr, const float* d_norm_w, float eps, int swiglu, float* d_ws,
                        void* stream) {
  if (!qw || !d_x || !d_y) return N730_NULL;
  N730_REQUIRE(tokens >= 1, N730_BAD_ARG, "qgemm: tokens %d", tokens);
  GemvArgs a = {};
  a.w = (const QWeight*)qw; a.x = d_x; a.ldx = ldx; a.batch = tokens; a.y = d_y; a.ldy = ldy;
  a.bias = d_bias; a.residual = d_residual; a.ldr = ldr; a.norm_w = d_norm_w; a.eps = eps; a.swiglu = swiglu;
  return gemm_tc_launch(a, d_ws, (cudaStream_t)stream);
}

N730_API int n730_quantize_grouped(const float* d_w, int rows, int cols, int bits, int group,
                                   uint8_t* d_codes, uint16_t* d_scales16, uint16_t* d_zeros16,
                                   void* stream) {
  if (!d_w || !d_codes || !d_scales16 || !d_zeros16) return N730_NULL;
  N730_REQUIRE(bits == 2 || bits == 4 || bits == 8, N730_BAD_ARG, "quantize: bits %d", bits);
  N730_REQUIRE(group > 0 && cols % group == 0 && group % (128 / bits) == 0, N730_BAD_ARG,
               "quantize: group %d invalid for INT%d cols=%d", group, bits, cols);
  cudaStream_t st = (cudaStream_t)stream;
  int* flag = nullptr;
  N730_CUDA(cudaMallocAsync(&flag, 4, st));
  N730_CUDA(cudaMemsetAsync(flag, 0, 4, st));
  const int64_t warps = (int64_t)rows * (cols / group);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, num_sms() * 32));
  quantize_grouped_kernel<<<grid, 256, 0, st>>>(d_w, rows, cols, bits, group, d_codes,
                                                (__half*)d_scales16, (__half*)d_zeros16, flag);
  N730_CHECK_LAUNCH();
  int h = 0;
  N730_CUDA(cudaMemcpyAsync(&h, flag, 4, cudaMemcpyDeviceToHost, st));
  N730_CUDA(cudaFreeAsync(flag, st));
  N730_CUDA(cudaStreamSynchronize(st));
  N730_REQUIRE(!h, N730_BAD_ARG, "quantize: a group scale overflows fp16");
  return N730_OK;
}
