// The reference's CUDA C ABI (src-code/cpp/n730_cuda.cu, 26 exported symbols,
// bound by src-code/inference.py:46-138 and src-code/diagnose_binary.py),
// re-implemented on this library's kernels so the reference's Python host
// layer loads this library unchanged.
//
// Semantics kept: implicit context buffers (d_activations, d_norm_buf,
// d_scores), fp32 activations, blocking calls on the legacy default stream,
// the same return codes.  Differences (all fixes): n730_upload_weight keeps the
// packed codes on the device and n730_linear runs the fused dequant-GEMV on
// them (no fp32 weight copy, no cuBLAS); INT2 and FP16 uploads decode
// correctly (the reference routes both through its INT8 kernel and over-reads
// the INT2 host buffer, n730_cuda.cu:483-501); byte counts are 64-bit.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "qweight.h"

namespace n730 {

struct LegacyCtx {
  int hidden, heads, head_dim, vocab, max_seq;
  int64_t max_w;
  float* d_activations = nullptr;   // [max_seq, hidden]
  float* d_norm_buf = nullptr;      // [max_seq, hidden]
  float* d_scores = nullptr;        // [heads, max_seq, max_seq]
  uint8_t* d_raw = nullptr;         // uploaded packed codes
  int64_t raw_cap = 0;
  uint8_t* d_rows = nullptr;        // codes repacked to 16-byte rows when needed
  int64_t rows_cap = 0;
  uint8_t* d_sz = nullptr;          // per-row (scale, zero), 16-byte rows, of the current weight
  int sz_cap = 0;
  int prec = 0;
  int64_t n_elements = 0;
  float scale = 1.f, zp = 0.f;
};

__global__ void rmsnorm_rows_kernel(const float* x, float* out, const float* w, int hidden, float eps) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * hidden;
  float* orow = out + (int64_t)blockIdx.x * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) ss += xr[i] * xr[i];
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) orow[i] = xr[i] * inv * w[i];
}

__global__ void axpy_kernel(float* x, const float* d, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += d[i];
}

__global__ void add_bias_kernel2(float* x, const float* b, int seq, int dim) {
  const int64_t n = (int64_t)seq * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += b[i % dim];
}

__global__ void swiglu_kernel(float* g, const float* u, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    g[i] = (x / (1.0f + expf(-x))) * u[i];
  }
}

// rotate_half RoPE, pos = s + offset (n730_cuda.cu:277-304)
__global__ void rope_f32_kernel(float* x, const float* cosf_, const float* sinf_, int seq, int heads,
                                int hd, int offset) {
  const int s = blockIdx.x, h = blockIdx.y, h2 = hd / 2;
  for (int i = threadIdx.x; i < h2; i += blockDim.x) {
    float* xs = x + ((int64_t)s * heads + h) * hd;
    const int pos = s + offset;
    const float c = cosf_[(int64_t)pos * h2 + i], sn = sinf_[(int64_t)pos * h2 + i];
    const float x0 = xs[i], x1 = xs[i + h2];
    xs[i] = x0 * c - x1 * sn;
    xs[i + h2] = x1 * c + x0 * sn;
  }
}

// scores[h, q, t] = scale * <Q[q, h, :], K[t, h/grp, :]>
__global__ void scores_kernel(const float* q, const float* k, float* sc, int seq_q, int seq_total,
                              int nh, int nkv, int hd, float scale) {
  extern __shared__ float qs[];
  const int qi = blockIdx.y, h = blockIdx.z, kvh = h / (nh / nkv);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) qs[d] = q[((int64_t)qi * nh + h) * hd + d];
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= seq_total) return;
  const float* kr = k + ((int64_t)t * nkv + kvh) * hd;
  float acc = 0.f;
  for (int d = 0; d < hd; ++d) acc += qs[d] * kr[d];
  sc[((int64_t)h * seq_q + qi) * seq_total + t] = acc * scale;
}

// causal mask (k > offset + q -> -1e4) and softmax exp(max(s - m, -50)) / (sum + 1e-9)
// (n730_cuda.cu:202-275)
__global__ void mask_softmax_kernel(float* sc, int seq_q, int seq_total, int offset, int mask) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int qi = row % seq_q;
  float* s = sc + (int64_t)row * seq_total;
  if (mask)
    for (int t = threadIdx.x; t < seq_total; t += blockDim.x)
      if (t > offset + qi) s[t] = -1e4f;
  __syncthreads();
  float mx = -1e20f;
  for (int t = threadIdx.x; t < seq_total; t += blockDim.x) mx = fmaxf(mx, s[t]);
  mx = warp_max(mx);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -1e20f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.f;
  for (int t = threadIdx.x; t < seq_total; t += blockDim.x) {
    const float e = expf(fmaxf(s[t] - mx, -50.0f));
    s[t] = e;
    sum += e;
  }
  sum = block_sum(sum, red) + 1e-9f;
  for (int t = threadIdx.x; t < seq_total; t += blockDim.x) s[t] /= sum;
}

// out[q, h*hd + d] = sum_t P[h, q, t] * V[t, h/grp, d]
__global__ void pv_kernel(const float* p, const float* v, float* out, int seq_q, int seq_total,
                          int nh, int nkv, int hd) {
  const int qi = blockIdx.x, h = blockIdx.y, kvh = h / (nh / nkv);
  const float* pr = p + ((int64_t)h * seq_q + qi) * seq_total;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < seq_total; ++t) acc += pr[t] * v[((int64_t)t * nkv + kvh) * hd + d];
    out[((int64_t)qi * nh + h) * hd + d] = acc;
  }
}

static int grid1(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, num_sms() * 8));
}

static int legacy_linear(LegacyCtx* c, const float* d_in, float* d_out, int seq, int in_dim, int out_dim) {
  N730_REQUIRE(c->d_raw && c->prec, N730_STATE, "n730_linear: no weight uploaded");
  N730_REQUIRE((int64_t)in_dim * out_dim == c->n_elements, N730_BAD_ARG,
               "n730_linear: %d x %d does not match the uploaded weight (%lld elements)", out_dim,
               in_dim, (long long)c->n_elements);
  const int bits = prec_bits(c->prec);
  QWeight w;
  w.prec = c->prec; w.bits = bits; w.rows = out_dim; w.cols = in_dim;
  w.group = in_dim; w.n_groups = 1; w.sz_mode = 1; w.owns = false;
  const int64_t rb = ((int64_t)in_dim * bits + 7) / 8;
  if (((int64_t)in_dim * bits) % 128 == 0) {
    w.codes = c->d_raw; w.row_bytes = rb;
  } else {
    w.row_bytes = (rb + 15) / 16 * 16;
    const int64_t need = w.row_bytes * out_dim;
    if (need > c->rows_cap) {
      cudaFree(c->d_rows);
      N730_CUDA(cudaMalloc(&c->d_rows, need));
      c->rows_cap = need;
    }
    if (int rc = repack_rows_launch(c->d_raw, bits, out_dim, in_dim, c->d_rows, w.row_bytes, 0)) return rc;
    w.codes = c->d_rows;
  }
  if (bits != 16) {
    if (out_dim > c->sz_cap) {
      cudaFree(c->d_sz);
      N730_CUDA(cudaMalloc(&c->d_sz, (size_t)out_dim * 16));
      c->sz_cap = out_dim;
    }
    if (int rc = fill_f2_launch(c->d_sz, 16, out_dim, c->scale, c->zp, 0)) return rc;
    w.sz = c->d_sz;
    w.sz_pitch = 16;
  }
  GemvArgs a = {};
  a.w = &w; a.x = d_in; a.ldx = in_dim; a.batch = seq; a.y = d_out; a.ldy = out_dim;
  return gemv_launch(a, 0);
}

}  // namespace n730

using namespace n730;

#define CTX(p) LegacyCtx* c = (LegacyCtx*)(p); if (!c) return N730_NULL

N730_API int n730_cuda_init(int hidden_size, int num_heads, int head_dim, int vocab_size, int max_seq,
                            int max_weight_elements, void** out_ctx) {
  if (!out_ctx) return N730_NULL;
  *out_ctx = nullptr;
  N730_REQUIRE(hidden_size > 0 && num_heads > 0 && max_seq > 0, N730_BAD_ARG, "n730_cuda_init: bad sizes");
  LegacyCtx* c = new LegacyCtx();
  c->hidden = hidden_size; c->heads = num_heads; c->head_dim = head_dim; c->vocab = vocab_size;
  c->max_seq = max_seq; c->max_w = max_weight_elements;
  const size_t ab = (size_t)max_seq * hidden_size * 4;
  const size_t sb = (size_t)num_heads * max_seq * max_seq * 4;
  if (cudaMalloc(&c->d_activations, ab) != cudaSuccess || cudaMalloc(&c->d_norm_buf, ab) != cudaSuccess ||
      cudaMalloc(&c->d_scores, sb) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(c->d_activations); cudaFree(c->d_norm_buf); cudaFree(c->d_scores);
    delete c;
    return N730_OOM;
  }
  *out_ctx = c;
  return N730_OK;
}

N730_API void n730_cuda_destroy(void* ctx) {
  LegacyCtx* c = (LegacyCtx*)ctx;
  if (!c) return;
  cudaFree(c->d_activations); cudaFree(c->d_norm_buf); cudaFree(c->d_scores);
  cudaFree(c->d_raw); cudaFree(c->d_rows); cudaFree(c->d_sz);
  delete c;
}

N730_API int n730_load_activations(void* ctx, const float* host, int seq, int hidden) {
  CTX(ctx);
  N730_REQUIRE(host && seq >= 0 && seq <= c->max_seq && hidden == c->hidden, N730_BAD_ARG,
               "load_activations: bad arguments");
  N730_CUDA(cudaMemcpy(c->d_activations, host, (size_t)seq * hidden * 4, cudaMemcpyHostToDevice));
  return N730_OK;
}

N730_API int n730_get_activations(void* ctx, float* host, int seq, int hidden) {
  CTX(ctx);
  N730_REQUIRE(host && seq >= 0 && seq <= c->max_seq && hidden == c->hidden, N730_BAD_ARG,
               "get_activations: bad arguments");
  N730_CUDA(cudaMemcpy(host, c->d_activations, (size_t)seq * hidden * 4, cudaMemcpyDeviceToHost));
  return N730_OK;
}

N730_API int n730_upload_weight(void* ctx, const uint8_t* raw, int prec_id, int n_elements, float scale,
                                float zero_point) {
  CTX(ctx);
  if (!raw) return N730_NULL;
  const int bits = prec_bits(prec_id);
  N730_REQUIRE(bits && !prec_grouped(prec_id), N730_BAD_ARG,
               "upload_weight: precision %d is not a per-tensor id", prec_id);
  N730_REQUIRE(n_elements > 0, N730_BAD_ARG, "upload_weight: n_elements %d", n_elements);
  const int64_t bytes = ((int64_t)n_elements * bits + 7) / 8;
  if (bytes > c->raw_cap) {
    cudaFree(c->d_raw);
    c->d_raw = nullptr;
    N730_CUDA(cudaMalloc(&c->d_raw, bytes));
    c->raw_cap = bytes;
  }
  N730_CUDA(cudaMemcpy(c->d_raw, raw, bytes, cudaMemcpyHostToDevice));
  c->prec = prec_id; c->n_elements = n_elements; c->scale = scale; c->zp = zero_point;
  return N730_OK;
}

N730_API int n730_upload_norm_weight(const float* host_w, int n, void** out_ptr) {
  if (!host_w || !out_ptr) return N730_NULL;
  float* d = nullptr;
  if (cudaMalloc(&d, (size_t)n * 4) != cudaSuccess) { cudaGetLastError(); return N730_OOM; }
  if (cudaMemcpy(d, host_w, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(d);
    return N730_CUDA_ERR;
  }
  *out_ptr = d;
  return N730_OK;
}

N730_API void n730_free_device_buf(void* p) { if (p) cudaFree(p); }

N730_API int n730_rmsnorm(void* ctx, const float* d_norm_w, int seq, float eps) {
  CTX(ctx);
  if (!d_norm_w) return N730_NULL;
  if (seq <= 0) return N730_OK;
  rmsnorm_rows_kernel<<<seq, 256>>>(c->d_activations, c->d_norm_buf, d_norm_w, c->hidden, eps);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_linear(void* ctx, float* d_out, int seq, int in_dim, int out_dim) {
  CTX(ctx);
  if (!d_out) return N730_NULL;
  return legacy_linear(c, c->d_norm_buf, d_out, seq, in_dim, out_dim);
}

N730_API int n730_linear_from_buf(void* ctx, const float* d_in, float* d_out, int seq, int in_dim, int out_dim) {
  CTX(ctx);
  if (!d_in || !d_out) return N730_NULL;
  return legacy_linear(c, d_in, d_out, seq, in_dim, out_dim);
}

N730_API int n730_residual_add(void* ctx, const float* d_delta, int seq) {
  CTX(ctx);
  if (!d_delta) return N730_NULL;
  const int64_t n = (int64_t)seq * c->hidden;
  if (n <= 0) return N730_OK;
  axpy_kernel<<<grid1(n), 256>>>(c->d_activations, d_delta, n);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_add_bias(void* ctx, float* d_out, const float* d_bias, int seq, int dim) {
  CTX(ctx);
  if (!d_out || !d_bias) return N730_NULL;
  const int64_t n = (int64_t)seq * dim;
  if (n <= 0) return N730_OK;
  add_bias_kernel2<<<grid1(n), 256>>>(d_out, d_bias, seq, dim);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_swiglu(float* d_gate, float* d_up, int seq, int inter) {
  if (!d_gate || !d_up) return N730_NULL;
  const int64_t n = (int64_t)seq * inter;
  if (n <= 0) return N730_OK;
  swiglu_kernel<<<grid1(n), 256>>>(d_gate, d_up, n);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_apply_rope(float* d_x, const float* d_cos, const float* d_sin, int seq, int heads,
                             int head_dim, int pos_off) {
  if (!d_x || !d_cos || !d_sin) return N730_NULL;
  if (seq <= 0 || heads <= 0) return N730_OK;
  rope_f32_kernel<<<dim3(seq, heads), std::min(std::max(head_dim / 2, 32), 256)>>>(
      d_x, d_cos, d_sin, seq, heads, head_dim, pos_off);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

// Host table exactly as n730_cuda.cu:650-661 (fp32 powf/cosf/sinf).
N730_API int n730_rope_precompute(int max_seq, int head_dim, float theta, void** d_cos_out, void** d_sin_out) {
  if (!d_cos_out || !d_sin_out) return N730_NULL;
  N730_REQUIRE(max_seq > 0 && head_dim > 0 && head_dim % 2 == 0, N730_BAD_ARG, "rope_precompute: bad sizes");
  const int h2 = head_dim / 2;
  const size_t n = (size_t)max_seq * h2;
  float* hc = new float[n];
  float* hs = new float[n];
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < h2; ++i) {
      const float freq = 1.0f / powf(theta, (float)(2 * i) / head_dim);
      const float angle = pos * freq;
      hc[(size_t)pos * h2 + i] = cosf(angle);
      hs[(size_t)pos * h2 + i] = sinf(angle);
    }
  float *dc = nullptr, *ds = nullptr;
  int rc = N730_OK;
  if (cudaMalloc(&dc, n * 4) != cudaSuccess || cudaMalloc(&ds, n * 4) != cudaSuccess) {
    cudaGetLastError(); cudaFree(dc); cudaFree(ds); rc = N730_OOM;
  } else if (cudaMemcpy(dc, hc, n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
             cudaMemcpy(ds, hs, n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(dc); cudaFree(ds); rc = N730_CUDA_ERR;
  } else {
    *d_cos_out = dc; *d_sin_out = ds;
  }
  delete[] hc; delete[] hs;
  return rc;
}

N730_API int n730_softmax_scores(float* d_scores, int heads, int seq_q, int seq_total, int cache_offset) {
  if (!d_scores) return N730_NULL;
  if (heads * seq_q <= 0 || seq_total <= 0) return N730_OK;
  mask_softmax_kernel<<<heads * seq_q, 128>>>(d_scores, seq_q, seq_total, cache_offset, seq_q > 1);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

static int attn_scores(LegacyCtx* c, const float* q, const float* k, int seq_q, int seq_total, int nh,
                       int nkv, int hd) {
  N730_REQUIRE(seq_q <= c->max_seq && seq_total <= c->max_seq && nh <= c->heads && nkv > 0 && nh % nkv == 0,
               N730_BAD_ARG, "attention: sizes exceed the context");
  scores_kernel<<<dim3((seq_total + 127) / 128, seq_q, nh), 128, hd * 4>>>(
      q, k, c->d_scores, seq_q, seq_total, nh, nkv, hd, 1.0f / sqrtf((float)hd));
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_attention_forward(void* ctx, const float* d_q, const float* d_k_cache, const float* d_v_cache,
                                    float* d_out, int seq_q, int seq_total, int n_heads, int n_kv_heads,
                                    int head_dim, int cache_offset) {
  CTX(ctx);
  if (!d_q || !d_k_cache || !d_v_cache || !d_out) return N730_NULL;
  if (seq_q <= 0 || seq_total <= 0) return N730_OK;
  if (int rc = attn_scores(c, d_q, d_k_cache, seq_q, seq_total, n_heads, n_kv_heads, head_dim)) return rc;
  mask_softmax_kernel<<<n_heads * seq_q, 128>>>(c->d_scores, seq_q, seq_total, cache_offset, seq_q > 1);
  N730_CHECK_LAUNCH();
  pv_kernel<<<dim3(seq_q, n_heads), std::min(head_dim, 256)>>>(c->d_scores, d_v_cache, d_out, seq_q,
                                                               seq_total, n_heads, n_kv_heads, head_dim);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

// ---------------------------------------------------------------------------
// No-allocation variant of n730_attention_forward (no counterpart in the
// reference).  Same kernels and results, but the [heads, seq_q, seq_total]
// score matrix lives in a fixed file-scope device array instead of the
// context's heads x max_seq^2 buffer, so the call needs no context, performs
// no cudaMalloc / cudaFree and cannot fail for lack of memory after start-up.
// For callers that must not allocate: a context sized for long contexts does
// not fit (64 heads x 8192^2 positions is 17 GB of scores), and cudaMalloc /
// cudaFree per call would synchronise the device under work on other streams.
//  * Limit: heads * seq_q * seq_total <= N730_ATTN_SCRATCH_FLOATS (1 Mi floats,
//    4 MiB; e.g. decode of 64 heads over 16384 positions), and seq_q, heads
//    <= 65535; larger requests return N730_BAD_ARG before any GPU work.
//  * The scratch address is resolved with cudaGetSymbolAddress once per device,
//    on that device's first call; make that first call outside stream capture.
//  * Nothing in the scratch must start at zero: scores_kernel writes every
//    element that the softmax and P V kernels read.
//  * One scratch per device: calls that overlap in time (other streams, other
//    host threads) race on it; serialise them.
// ---------------------------------------------------------------------------
constexpr int64_t N730_ATTN_SCRATCH_FLOATS = int64_t(1) << 20;
static __device__ __align__(256) float g_attn_scratch[N730_ATTN_SCRATCH_FLOATS];

static float* attn_scratch(int dev) {
  static std::mutex mu;
  static float* addr[128] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  return addr[dev];
}

N730_API int n730_attention_forward_noalloc(const float* d_q, const float* d_k_cache, const float* d_v_cache,
                                            float* d_out, int seq_q, int seq_total, int n_heads, int n_kv_heads,
                                            int head_dim, int cache_offset, void* stream) {
  if (!d_q || !d_k_cache || !d_v_cache || !d_out) return N730_NULL;
  if (seq_q <= 0 || seq_total <= 0) return N730_OK;
  N730_REQUIRE(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0 && head_dim > 0 && head_dim <= 4096,
               N730_BAD_ARG, "attention_noalloc: bad heads / head_dim");
  N730_REQUIRE((int64_t)n_heads * seq_q * seq_total <= N730_ATTN_SCRATCH_FLOATS, N730_BAD_ARG,
               "attention_noalloc: %d heads x %d x %d scores exceed the %lld-float scratch", n_heads, seq_q,
               seq_total, (long long)N730_ATTN_SCRATCH_FLOATS);
  // seq_q and n_heads index grid.y / grid.z of the score and P V launches (at most 65535 each)
  N730_REQUIRE(seq_q <= 65535 && n_heads <= 65535, N730_BAD_ARG,
               "attention_noalloc: seq_q %d / heads %d exceed the 65535 launch-grid limit", seq_q, n_heads);
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < 128, N730_BAD_ARG, "attention_noalloc: device %d", dev);
  float* sc = attn_scratch(dev);
  N730_REQUIRE(sc, N730_CUDA_ERR, "attention_noalloc: scratch address unavailable");
  cudaStream_t st = (cudaStream_t)stream;
  scores_kernel<<<dim3((seq_total + 127) / 128, seq_q, n_heads), 128, head_dim * 4, st>>>(
      d_q, d_k_cache, sc, seq_q, seq_total, n_heads, n_kv_heads, head_dim, 1.0f / sqrtf((float)head_dim));
  N730_CHECK_LAUNCH();
  mask_softmax_kernel<<<n_heads * seq_q, 128, 0, st>>>(sc, seq_q, seq_total, cache_offset, seq_q > 1);
  N730_CHECK_LAUNCH();
  pv_kernel<<<dim3(seq_q, n_heads), std::min(head_dim, 256), 0, st>>>(sc, d_v_cache, d_out, seq_q, seq_total,
                                                                     n_heads, n_kv_heads, head_dim);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

N730_API int n730_attention_qk_only(void* ctx, const float* d_q, const float* d_k_cache, int seq_q, int seq_total,
                                    int n_heads, int n_kv_heads, int head_dim) {
  CTX(ctx);
  if (!d_q || !d_k_cache) return N730_NULL;
  if (seq_q <= 0 || seq_total <= 0) return N730_OK;
  return attn_scores(c, d_q, d_k_cache, seq_q, seq_total, n_heads, n_kv_heads, head_dim);
}

N730_API int n730_get_scores(void* ctx, float* host, int n_heads, int seq_q, int seq_total) {
  CTX(ctx);
  if (!host) return N730_NULL;
  N730_CUDA(cudaMemcpy(host, c->d_scores, (size_t)n_heads * seq_q * seq_total * 4, cudaMemcpyDeviceToHost));
  return N730_OK;
}

N730_API int n730_device_alloc(int n_floats, void** out_ptr) {
  if (!out_ptr) return N730_NULL;
  float* p = nullptr;
  if (cudaMalloc(&p, (size_t)n_floats * 4) != cudaSuccess) { cudaGetLastError(); return N730_OOM; }
  *out_ptr = p;
  return N730_OK;
}

N730_API void n730_device_free(void* p) { if (p) cudaFree(p); }

N730_API int n730_memcpy_d2d(void* dst, const void* src, int n_floats) {
  N730_CUDA(cudaMemcpy(dst, src, (size_t)n_floats * 4, cudaMemcpyDeviceToDevice));
  return N730_OK;
}
N730_API int n730_memcpy_h2d(void* dst, const void* src, int n_floats) {
  N730_CUDA(cudaMemcpy(dst, src, (size_t)n_floats * 4, cudaMemcpyHostToDevice));
  return N730_OK;
}
N730_API int n730_memcpy_d2h(void* dst, const void* src, int n_floats) {
  N730_CUDA(cudaMemcpy(dst, src, (size_t)n_floats * 4, cudaMemcpyDeviceToHost));
  return N730_OK;
}

N730_API int n730_sync(void) {
  N730_CUDA(cudaDeviceSynchronize());
  return N730_OK;
}

N730_API const char* n730_cuda_version(void) {
  return "N730 B200 kernels 0.1 / sm_100a";
}
