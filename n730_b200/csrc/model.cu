// Whole-model engine: resident packed weights, paged fp16 KV cache, one-call
// decode step replayed as a CUDA graph, and prefill.
//
// Replaces the reference's per-op Python -> ctypes loop of
// N730CudaTransformer.forward (src-code/inference.py:467-669): per token it
// re-read every weight from disk, uploaded it synchronously, dequantised it to
// fp32, ran cuBLAS, and computed the final norm and lm_head on the CPU.  Here
// a decode step for B sequences is ~5 kernels per layer:
//   qkv GEMV (RMSNorm prologue, bias) -> RoPE+GQA decode attention (KV append,
//   split merge) -> o_proj GEMV (+residual) -> gate|up GEMV (RMSNorm, SwiGLU)
//   -> down GEMV (+residual)
// then the final-norm + lm_head GEMV and a position update, captured once per
// batch size into a CUDA graph whose kernels chain with programmatic dependent
// launch.  Host I/O per step is the token ids in and the logits out.
#include <array>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include <nccl.h>

#include "attention.h"
#include "decode_persist.h"
#include "tp_allreduce.h"
#include "n730_cuda.h"
#include "qweight.h"

namespace n730 {

int qweight_alloc_like(const QWeight& proto, int rows, QWeight** out);
int qweight_copy_rows(QWeight& dst, const QWeight& src, int dst_row0, int stride, cudaStream_t st);
void qweight_destroy(QWeight* w);

// x += d (the residual add after a tensor-parallel allreduce of the partial sums)
__global__ void add_inplace_kernel(float* x, const float* d, int64_t n) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += d[i];
}

// all-gathered vocab shards [T][B][vl] -> logits [B][T * vl]
__global__ void gather_logits_kernel(const float* all, float* out, int T, int B, int vl) {
  const int64_t n = (int64_t)T * B * vl;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % vl);
    const int64_t tb = i / vl;
    const int b = (int)(tb % B), t = (int)(tb / B);
    out[(int64_t)b * T * vl + (int64_t)t * vl + v] = all[i];
  }
}

__global__ void advance_seq_kernel(int* seq_lens, int batch, int by) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) seq_lens[b] += by;
}

struct Layer {
  QWeight* qkv = nullptr;
  QWeight* o = nullptr;
  QWeight* gate_up = nullptr;
  QWeight* down = nullptr;
  float* ln1 = nullptr;
  float* ln2 = nullptr;
  float* qkv_bias = nullptr;
  float* o_bias = nullptr;
  float* gate_up_bias = nullptr;
  float* down_bias = nullptr;
  KVLayer kv{};
};

struct Model {
  N730ModelConfig c{};
  int qkv_dim = 0;
  bool finalized = false;
  std::vector<Layer> L;
  std::map<std::pair<int, int>, QWeight*> pend_w;
  std::map<std::pair<int, int>, std::vector<float>> pend_v;
  QWeight* embed = nullptr;
  QWeight* lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<void*> allocs;
  float *cos_t = nullptr, *sin_t = nullptr;
  __half *k_pool = nullptr, *v_pool = nullptr;
  int* block_table = nullptr;
  int* seq_lens = nullptr;
  std::vector<int> h_seq;
  int max_pages = 0, n_split = 1;
  // paged KV pool: pages are handed to a sequence as its length grows and returned when it is
  // released; h_bt mirrors the device block table [max_batch][max_pages]
  std::vector<int> free_pages;
  std::vector<std::vector<int>> seq_pages;
  std::vector<int> h_bt;
  int pool_pages = 0;
  // decode workspace
  int* d_tokens = nullptr;
  float *x = nullptr, *x2 = nullptr, *qkv = nullptr, *attn = nullptr, *mlp = nullptr, *logits = nullptr;
  // prefill workspace
  int* p_tokens = nullptr;
  float *px = nullptr, *pqkv = nullptr, *pattn = nullptr, *pmlp = nullptr;
  int32_t* h_tok = nullptr;  // pinned
  float* h_logits = nullptr;  // pinned [max_batch][vocab]
  cudaStream_t st = nullptr;
  std::map<int, cudaGraphExec_t> graphs;
  int device = 0;
  // persistent batch-1 decode (decode_persist.cu)
  bool pd_ok = false;
  bool plan_mismatch = false;
  int32_t* d_next = nullptr;      // GPU sampling: [max_batch] next-token ids, then [max_batch] u draws
  unsigned long long sample_steps = 0;  // sampled decode steps (the counter of the draws)
  std::vector<int8_t> pd_kinds;   // the persistent plan's phase kinds (PD_GEMV / PD_ATTN / PD_FFN), host copy
  unsigned long long* pd_trace = nullptr;  // per-phase timing buffer (n730_model_trace_step)    // tensor parallel: the ranks' persistent plans differed (per-op path)
  bool pd_ffn_fused = false;     // the persistent step runs each FFN as one phase
  std::map<const QWeight*, uint8_t*> pd_tiles;  // INT8 / FP16 weights as persistent-kernel tiles
  std::map<const QWeight*, uint8_t*> pd_down_gm;  // fused FFN: down_proj tiles in group-major order
  PdPlan pd;
  // layer streaming (stream_depth > 0): per-layer weight images in pinned host
  // memory, copied into HBM slots on `cst` ahead of use
  struct WOff { int64_t codes, sz; };
  std::vector<uint8_t*> img;                 // [layers] pinned host images
  std::vector<int64_t> img_bytes;            // [layers]
  std::vector<std::array<WOff, 4>> img_off;  // [layers][qkv, o, gate_up, down]
  std::vector<uint8_t*> slot;                // [depth + 1] HBM slots
  std::vector<std::array<QWeight, 4>> slot_w;  // weights bound to a slot
  std::vector<cudaEvent_t> ev_ready, ev_free;  // per slot
  cudaStream_t cst = nullptr;
  int64_t streamed_bytes = 0;                // host->HBM bytes per forward pass
  // tensor parallel (tp_size > 1): partial sums of the row-split o/down
  // projections are allreduced before the residual add; the lm_head is split
  // by vocabulary and its logits all-gathered
  ncclComm_t comm = nullptr;
  float* delta = nullptr;        // [max(max_batch, max_prefill)][hidden]
  float* logits_all = nullptr;   // [tp][max_batch][vocab / tp]
  int vocab_l = 0;               // lm_head rows on this rank
  float* rms_ws = nullptr;       // [max(max_batch, max_prefill)] per-token 1/rms for the tcgen05 GEMM
  // sums of squares of the residual stream left by the split-K fold of the o_proj / down_proj GEMM
  // that last wrote it ([max(max_batch, max_prefill)][ceil(hidden / TC_SS_ROWS)]); the next
  // RMSNorm'd GEMM reads them instead of a pass over x.  ss_of / ss_rows name the x and the rows
  // they describe while a forward is enqueued; any other launch clears ss_of.
  float* ss_ws = nullptr;
  const float* ss_of = nullptr;
  int ss_rows = 0;
  float* split_ws = nullptr;     // split-K partial sums of batched GEMVs [16][min(max_batch, 16)][hidden]
  int64_t split_ws_floats = 0;
  unsigned long long* ffn_acc = nullptr;  // persistent decode, fused FFN: [hidden] down_proj sums (fixed point)
  // one-shot peer-memory allreduce (tp_allreduce.cu): this rank's exchange
  // region, the peers' regions mapped with CUDA IPC, the op counters
  void* ar_base = nullptr;
  std::vector<void*> ar_peer_base;
  ArArgs ar{};
  bool ar_ok = false;
  bool ar_off = false;           // a peer-memory exchange timed out: NCCL for the rest of the model's life

  template <typename T>
  int alloc(T** p, size_t n) {
    void* q = nullptr;
    if (cudaMalloc(&q, n * sizeof(T)) != cudaSuccess) {
      cudaGetLastError();
      set_error("model: out of device memory allocating %zu bytes", n * sizeof(T));
      return N730_OOM;
    }
    allocs.push_back(q);
    *p = (T*)q;
    return N730_OK;
  }
};

static int upload_vec(Model* m, const std::vector<float>& v, float** out) {
  if (int rc = m->alloc(out, v.size())) return rc;
  N730_CUDA(cudaMemcpyAsync(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice, m->st));
  return N730_OK;
}

static int fuse_rows(Model* m, std::vector<QWeight*> parts, bool interleave, QWeight** out) {
  for (auto* p : parts) N730_REQUIRE(p, N730_STATE, "model: missing projection weight");
  int rows = 0;
  for (auto* p : parts) rows += p->rows;
  QWeight* f = nullptr;
  if (int rc = qweight_alloc_like(*parts[0], rows, &f)) return rc;
  int r0 = 0;
  for (size_t i = 0; i < parts.size(); ++i) {
    int rc = interleave ? qweight_copy_rows(*f, *parts[i], (int)i, (int)parts.size(), m->st)
                        : qweight_copy_rows(*f, *parts[i], r0, 1, m->st);
    if (rc) { qweight_destroy(f); return rc; }
    r0 += parts[i]->rows;
  }
  *out = f;
  return N730_OK;
}

static AttnDims dims(const Model* m);

static int64_t dev_code_bytes(const QWeight* w) {
  if (w->layout == 1) return (int64_t)((w->rows + 15) / 16) * w->n_groups * ((int64_t)(w->group / 16) * 128 + 64);
  return (int64_t)w->rows * w->row_bytes;
}
static int64_t dev_sz_bytes(const QWeight* w) {
  return (w->layout == 1 || w->bits == 16) ? 0 : (int64_t)w->rows * w->sz_pitch;
}

// Move every layer's weights into a pinned host image (after fusion and layout
// conversion, so an image is the exact device bytes) and set up the HBM slots.
static int setup_streaming(Model* m) {
  const int nl = m->c.layers, ns = m->c.stream_depth + 1;
  m->img.assign(nl, nullptr);
  m->img_bytes.assign(nl, 0);
  m->img_off.assign(nl, {});
  int64_t slot_bytes = 0;
  for (int l = 0; l < nl; ++l) {
    Layer& y = m->L[l];
    QWeight* ws[4] = {y.qkv, y.o, y.gate_up, y.down};
    int64_t off = 0;
    for (int k = 0; k < 4; ++k) {
      m->img_off[l][k].codes = off;
      off += (dev_code_bytes(ws[k]) + 255) / 256 * 256;
      m->img_off[l][k].sz = off;
      off += (dev_sz_bytes(ws[k]) + 255) / 256 * 256;
    }
    m->img_bytes[l] = off;
    slot_bytes = std::max(slot_bytes, off);
    N730_CUDA(cudaMallocHost(&m->img[l], off));
    for (int k = 0; k < 4; ++k) {
      QWeight* w = ws[k];
      N730_CUDA(cudaMemcpy(m->img[l] + m->img_off[l][k].codes, w->codes, dev_code_bytes(w), cudaMemcpyDeviceToHost));
      if (dev_sz_bytes(w))
        N730_CUDA(cudaMemcpy(m->img[l] + m->img_off[l][k].sz, w->sz, dev_sz_bytes(w), cudaMemcpyDeviceToHost));
      if (w->owns) { cudaFree(w->codes); cudaFree(w->sz); }
      w->codes = nullptr;  // metadata only from here on
      w->sz = nullptr;
      w->owns = false;
    }
    m->streamed_bytes += off;
  }
  m->slot.assign(ns, nullptr);
  m->slot_w.assign(ns, {});
  m->ev_ready.assign(ns, nullptr);
  m->ev_free.assign(ns, nullptr);
  for (int s = 0; s < ns; ++s) {
    if (int rc = m->alloc(&m->slot[s], (size_t)slot_bytes)) return rc;
    N730_CUDA(cudaEventCreateWithFlags(&m->ev_ready[s], cudaEventDisableTiming));
    N730_CUDA(cudaEventCreateWithFlags(&m->ev_free[s], cudaEventDisableTiming));
    N730_CUDA(cudaEventRecord(m->ev_free[s], m->st));
  }
  N730_CUDA(cudaStreamCreateWithFlags(&m->cst, cudaStreamNonBlocking));
  return N730_OK;
}

// Copy layer l's image into its slot on the copy stream, after the slot's
// previous layer has finished computing.
static int stream_issue(Model* m, int l) {
  const int s = l % (int)m->slot.size();
  N730_CUDA(cudaStreamWaitEvent(m->cst, m->ev_free[s], 0));
  N730_CUDA(cudaMemcpyAsync(m->slot[s], m->img[l], (size_t)m->img_bytes[l], cudaMemcpyHostToDevice, m->cst));
  N730_CUDA(cudaEventRecord(m->ev_ready[s], m->cst));
  return N730_OK;
}

struct LayerW { const QWeight *qkv, *o, *gate_up, *down; };

// Start of a pass over the layers: prefetch the first `depth` layers.
static int stream_begin(Model* m) {
  if (!m->c.stream_depth) return N730_OK;
  for (int l = 0; l < std::min(m->c.stream_depth, m->c.layers); ++l)
    if (int rc = stream_issue(m, l)) return rc;
  return N730_OK;
}

// Weights of layer l, ready to use on m->st (streamed: wait for its copy).
static int stream_acquire(Model* m, int l, LayerW* out) {
  Layer& y = m->L[l];
  if (!m->c.stream_depth) { *out = LayerW{y.qkv, y.o, y.gate_up, y.down}; return N730_OK; }
  const int s = l % (int)m->slot.size();
  N730_CUDA(cudaStreamWaitEvent(m->st, m->ev_ready[s], 0));
  const QWeight* meta[4] = {y.qkv, y.o, y.gate_up, y.down};
  for (int k = 0; k < 4; ++k) {
    QWeight& w = m->slot_w[s][k];
    w = *meta[k];
    w.codes = m->slot[s] + m->img_off[l][k].codes;
    w.sz = dev_sz_bytes(meta[k]) ? m->slot[s] + m->img_off[l][k].sz : nullptr;
    w.owns = false;
  }
  *out = LayerW{&m->slot_w[s][0], &m->slot_w[s][1], &m->slot_w[s][2], &m->slot_w[s][3]};
  return N730_OK;
}

// Layer l's kernels are enqueued: free its slot and start the copy `depth` layers ahead.
static int stream_release(Model* m, int l) {
  if (!m->c.stream_depth) return N730_OK;
  N730_CUDA(cudaEventRecord(m->ev_free[l % (int)m->slot.size()], m->st));
  if (l + m->c.stream_depth < m->c.layers) return stream_issue(m, l + m->c.stream_depth);
  return N730_OK;
}

// Phase table + scratch for the persistent batch-1 decode kernel.  Leaves
// pd_ok false (per-op kernels) when a weight is not in fragment tiles, groups
// differ, or the shapes exceed the kernel's limits.
constexpr int64_t PD_AUTO_MIN_LAYER_BYTES = 32ll << 20;

static int plan_persistent(Model* m) {
  const N730ModelConfig& c = m->c;
  if (c.stream_depth > 0) return N730_OK;  // weights not resident
  if (c.per_op_decode == 0) {  // auto: small layers decode faster through the per-op kernels
    int64_t b = 0;
    for (auto& y : m->L)
      for (const QWeight* w : {y.qkv, y.o, y.gate_up, y.down}) b += dev_code_bytes(w) + dev_sz_bytes(w);
    if (b < (int64_t)c.layers * PD_AUTO_MIN_LAYER_BYTES) return N730_OK;
  }
  // tensor parallel: the row-split sums cross over the mapped peer exchange regions
  const bool tp = c.tp_size > 1;
  if (tp && !(m->ar_ok && c.tp_size <= PD_MAX_RANKS && m->ar.cap >= c.hidden)) return N730_OK;
  // INT4 in fragment tiles stream as they are; INT8 (any scale/zero layout) and
  // FP16 weights get a tiled copy for the persistent kernel (decode_persist.h)
  auto tiled = [](const QWeight* w) { return w && w->layout == 1; };
  auto tileable = [&](const QWeight* w) {
    return w && (tiled(w) || ((w->bits == 8 || w->bits == 16) && w->layout == 0 && w->cols % PD_TILE_K == 0 &&
                              (w->bits == 16 || w->sz_mode == 1 || w->group % PD_TILE_K == 0)));
  };
  for (auto& y : m->L)
    if (!tileable(y.qkv) || !tileable(y.o) || !tiled(y.gate_up) || !tiled(y.down)) return N730_OK;
  if (!tileable(m->lm_head)) return N730_OK;
  auto make_tiles = [&](const QWeight* w) -> int {
    if (tiled(w) || m->pd_tiles.count(w)) return N730_OK;
    uint8_t* t = nullptr;
    if (int r = m->alloc(&t, (size_t)pd_tile_bytes(w->bits, w->rows, w->cols))) return r;
    if (int r = pd_tile_launch(*w, t, m->st)) return r;
    m->pd_tiles[w] = t;
    return N730_OK;
  };
  for (auto& y : m->L)
    for (const QWeight* w : {y.qkv, y.o})
      if (int r = make_tiles(w)) return r;
  if (int r = make_tiles(m->lm_head)) return r;
  int grid = 0;
  if (int r = persist_grid(&grid)) return r;
  const int g_down = m->L[0].down->n_groups;
  std::vector<PdPhase> ph;
  auto gemv_phase = [&](const QWeight* w, const float* x, const float* norm, const float* bias, float* y, int epi) {
    PdPhase p = {};
    p.kind = PD_GEMV; p.epi = epi; p.blob = w->codes; p.rows = w->rows; p.cols = w->cols; p.G = w->n_groups;
    p.prec = 4;
    if (!tiled(w)) { p.blob = m->pd_tiles.at(w); p.G = w->cols / PD_TILE_K; p.prec = (int8_t)w->bits; }
    p.x = x; p.norm_w = norm; p.bias = bias; p.y = y;
    ph.push_back(p);
  };
  // Fused FFN: the residual stream is h (m->x) + acc between a layer's FFN and
  // the next layer's o_proj, which folds acc into h and clears it; q|k|v and
  // the lm_head read h + acc.  Layers without a bias on down_proj only.
  // Tensor parallel (tp): q|k|v and gate|up are this rank's columns, o_proj and
  // down_proj its K columns.  Each of those row-split GEMVs pushes its partial
  // sums into every rank's exchange slot (parity e & 1 for exchange e); after
  // the cross-GPU barrier the next norm GEMV reads x = h + the ranks' sums in
  // rank order and writes the new residual to the other h buffer.  The bias of
  // a row-split projection is added on rank 0 only.
  auto build_tp = [&]() {
    ph.clear();
    float* hb[2] = {m->x, m->x2};
    int cur = 0, e = 0, xb = 0;
    auto xsum = [&](PdPhase& p, bool write_h) {
      p.x = hb[cur]; p.xsum = 1; p.xpar = (e - 1) & 1; p.xbar = ++xb;
      p.h_out = write_h ? hb[cur ^ 1] : nullptr;
      cur ^= 1;
    };
    const bool r0 = c.tp_rank == 0;
    for (int l = 0; l < c.layers; ++l) {
      const Layer& y = m->L[l];
      gemv_phase(y.qkv, hb[cur], y.ln1, y.qkv_bias, m->qkv, PD_EPI_STORE);
      if (l > 0) xsum(ph.back(), true);
      PdPhase at = {};
      at.kind = PD_ATTN; at.kv = y.kv;
      ph.push_back(at);
      gemv_phase(y.o, m->attn, nullptr, r0 ? y.o_bias : nullptr, nullptr, PD_EPI_XPUSH);
      ph.back().xpar = e++ & 1;
      gemv_phase(y.gate_up, hb[cur], y.ln2, y.gate_up_bias, m->mlp, PD_EPI_SWIGLU);
      xsum(ph.back(), true);
      gemv_phase(y.down, m->mlp, nullptr, r0 ? y.down_bias : nullptr, nullptr, PD_EPI_XPUSH);
      ph.back().xpar = e++ & 1;
    }
    float* lg = m->vocab_l == c.vocab ? m->logits : m->logits_all + (size_t)c.tp_rank * m->vocab_l;
    gemv_phase(m->lm_head, hb[cur], m->final_norm, nullptr, lg, PD_EPI_STORE);
    xsum(ph.back(), false);
    return xb;
  };
  auto build = [&](bool fuse) {
    ph.clear();
    unsigned long long* acc = fuse ? m->ffn_acc : nullptr;
    for (auto& y : m->L) {
      gemv_phase(y.qkv, m->x, y.ln1, y.qkv_bias, m->qkv, PD_EPI_STORE);
      ph.back().acc = acc;
      PdPhase at = {};
      at.kind = PD_ATTN; at.kv = y.kv;
      ph.push_back(at);
      gemv_phase(y.o, m->attn, nullptr, y.o_bias, m->x, PD_EPI_RESID);
      ph.back().acc = acc;
      gemv_phase(y.gate_up, m->x, y.ln2, y.gate_up_bias, m->mlp, PD_EPI_SWIGLU);
      if (fuse) {  // gate|up + down partial sums in one phase
        PdPhase& f = ph.back();
        f.kind = PD_FFN;
        f.blob2 = m->pd_down_gm.count(y.down) ? m->pd_down_gm.at(y.down) : nullptr; f.rows2 = y.down->rows; f.cols2 = y.down->cols; f.G2 = y.down->n_groups;
        f.acc = acc;
      } else {
        gemv_phase(y.down, m->mlp, nullptr, y.down_bias, m->x, PD_EPI_RESID);
      }
    }
    gemv_phase(m->lm_head, m->x, m->final_norm, nullptr, m->logits, PD_EPI_STORE);
    ph.back().acc = acc;
  };
  // the fused FFN streams down_proj from a group-major copy of its tiles (made once, kept)
  auto prep_down_gm = [&]() -> int {
    for (auto& y : m->L) {
      if (m->pd_down_gm.count(y.down)) continue;
      uint8_t* t = nullptr;
      const QWeight* w = y.down;
      const size_t bytes = (size_t)((w->rows + 15) / 16) * w->n_groups * ((size_t)(w->group / 16) * 128 + 64);
      if (int r = m->alloc(&t, bytes)) return r;
      if (int r = pd_group_major_launch(w->codes, w->rows, w->n_groups, w->group, t, m->st)) return r;
      m->pd_down_gm[w] = t;
    }
    return N730_OK;
  };
  bool has_down_bias = false;
  for (auto& y : m->L) has_down_bias |= y.down_bias != nullptr;
  bool fuse = !tp && !has_down_bias && (c.ffn_fuse > 0 || (c.ffn_fuse == 0 && g_down % grid == 0));
  if (tp && !m->x2)
    if (int r = m->alloc(&m->x2, (size_t)c.hidden)) return r;
  if (fuse && !m->ffn_acc) {
    if (int r = m->alloc(&m->ffn_acc, (size_t)c.hidden)) return r;
    N730_CUDA(cudaMemsetAsync(m->ffn_acc, 0, (size_t)c.hidden * 8, m->st));
  }
  PdPlan plan;
  int n_xbar = 0;
  if (fuse)
    if (int r = prep_down_gm()) return r;
  if (tp) n_xbar = build_tp();
  else build(fuse);
  int rc = persist_plan(ph.data(), (int)ph.size(), c.head_dim, c.heads / c.kv_heads, c.page_size, c.tp_size, &plan);
  if (rc == N730_UNSUPPORTED && fuse) {  // shapes outside the fused phase's limits: two GEMV phases
    fuse = false;
    build(false);
    rc = persist_plan(ph.data(), (int)ph.size(), c.head_dim, c.heads / c.kv_heads, c.page_size, c.tp_size, &plan);
  } else if (rc == N730_UNSUPPORTED && !tp && !has_down_bias && c.ffn_fuse == 0) {
    // auto mode, uneven down groups per SM: the two-phase FFN did not fit (down_proj's x in shared
    // memory, 72B: 29568 fp16), the fused one still runs persistently (faster than per-op kernels)
    fuse = true;
    if (!m->ffn_acc) {
      if (int r = m->alloc(&m->ffn_acc, (size_t)c.hidden)) return r;
      N730_CUDA(cudaMemsetAsync(m->ffn_acc, 0, (size_t)c.hidden * 8, m->st));
    }
    if (int r = prep_down_gm()) return r;
    build(true);
    rc = persist_plan(ph.data(), (int)ph.size(), c.head_dim, c.heads / c.kv_heads, c.page_size, c.tp_size, &plan);
  }
  if (rc == N730_UNSUPPORTED) return N730_OK;
  if (rc) return rc;
  m->pd_ffn_fused = fuse;
  plan.a.acc = fuse ? m->ffn_acc : nullptr;
  plan.a.acc_n = fuse ? c.hidden : 0;
  const int GQ = c.heads / c.kv_heads;
  const int max_split = std::min(64, plan.grid / c.kv_heads);
  if (max_split < 1) return N730_OK;
  PdArgs& a = plan.a;
  PdPhase* d_ph = nullptr;
  if (int r = m->alloc(&d_ph, ph.size())) return r;
  N730_CUDA(cudaMemcpyAsync(d_ph, ph.data(), ph.size() * sizeof(PdPhase), cudaMemcpyHostToDevice, m->st));
  a.phases = d_ph;
  a.n_phases = (int)ph.size();
  a.eps = c.rms_eps;
  a.qkv = m->qkv; a.attn_out = m->attn; a.cos_t = m->cos_t; a.sin_t = m->sin_t;
  a.seq_lens = m->seq_lens; a.block_table = m->block_table; a.d = dims(m);
  a.max_split = max_split;
  a.trace = nullptr;
  m->pd_kinds.clear();
  for (const PdPhase& q : ph) m->pd_kinds.push_back(q.kind);
  if (int r = m->alloc(&a.attn_part, (size_t)c.kv_heads * max_split * GQ * (c.head_dim + 2))) return r;
  if (int r = m->alloc(&a.attn_cnt, (size_t)c.kv_heads)) return r;
  if (int r = m->alloc(&a.sync, 4)) return r;
  N730_CUDA(cudaMemsetAsync(a.attn_cnt, 0, c.kv_heads * 4, m->st));
  N730_CUDA(cudaMemsetAsync(a.sync, 0, 16, m->st));
  a.err = gemv_err_word();
  if (tp) {
    a.tp_rank = c.tp_rank;
    a.tp_size = c.tp_size;
    a.xcap = m->ar.cap;
    for (int r = 0; r < c.tp_size; ++r) {
      a.xrecv[r] = m->ar.peer[r].recv;
      a.xcnt[r] = m->ar.peer[r].xcnt;
    }
    a.xrecv_local = a.xrecv[c.tp_rank];
    a.xcnt_local = a.xcnt[c.tp_rank];
    a.n_xbar = n_xbar;
    if (int r = m->alloc(&a.xepoch, 1)) return r;
    N730_CUDA(cudaMemsetAsync(a.xepoch, 0, 4, m->st));
  }
  N730_REQUIRE(a.err, N730_OOM, "model: error word allocation failed");
  m->pd = plan;
  m->pd_ok = true;
  return N730_OK;
}

// Tensor parallel: every rank must take the same batch-1 decode path.  The
// persistent kernel's cross-GPU barriers count tp_size x grid arrivals per
// barrier and its exchanges follow the phase table, so ranks that planned
// differently (another SM count, a persistent plan on one rank only, another
// number of phases) would pass barriers early or wait on a peer that runs the
// per-op kernels.  The ranks all-gather (persistent, grid, cross barriers,
// phases); unless all agree, every rank drops to the per-op path (NCCL), the
// same decision on every rank.
static int agree_decode_path(Model* m) {
  const N730ModelConfig& c = m->c;
  N730_REQUIRE(m->comm, N730_STATE, "model: tensor parallel finalize before tp_init");
  const int sig[4] = {m->pd_ok ? 1 : 0, m->pd_ok ? m->pd.grid : 0, m->pd_ok ? m->pd.a.n_xbar : 0,
                      m->pd_ok ? m->pd.a.n_phases : 0};
  int* d = nullptr;
  if (int rc = m->alloc(&d, (size_t)4 * (c.tp_size + 1))) return rc;
  N730_CUDA(cudaMemcpyAsync(d, sig, sizeof sig, cudaMemcpyHostToDevice, m->st));
  if (ncclAllGather(d, d + 4, 4, ncclInt32, m->comm, m->st) != ncclSuccess) {
    set_error("model: ncclAllGather of the decode plans failed");
    return N730_COMM;
  }
  std::vector<int> all((size_t)4 * c.tp_size);
  N730_CUDA(cudaMemcpyAsync(all.data(), d + 4, all.size() * 4, cudaMemcpyDeviceToHost, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  for (int r = 1; r < c.tp_size; ++r)
    if (memcmp(&all[4 * r], &all[0], 16) != 0) {
      m->pd_ok = false;
      m->plan_mismatch = true;
      break;
    }
  return N730_OK;
}

static int finalize(Model* m) {
  const N730ModelConfig& c = m->c;
  if (int rc = gemv_prepare()) return rc;
  if (int rc = gemm_tc_prepare()) return rc;
  if (int rc = gemm_tc_reserve(std::max(c.max_batch, c.max_prefill), std::max(c.hidden, c.ffn),
                               std::max(c.hidden, (c.heads + 2 * c.kv_heads) * c.head_dim), m->st))
    return rc;
  const int nl = c.layers;
  m->L.assign(nl, Layer{});
  auto W = [&](int l, int s) -> QWeight* {
    auto it = m->pend_w.find({l, s});
    return it == m->pend_w.end() ? nullptr : it->second;
  };
  auto V = [&](int l, int s) -> const std::vector<float>* {
    auto it = m->pend_v.find({l, s});
    return it == m->pend_v.end() ? nullptr : &it->second;
  };
  m->embed = W(-1, N730_W_EMBED);
  N730_REQUIRE(m->embed, N730_STATE, "model: embedding weight not set");
  N730_REQUIRE(m->embed->rows == c.vocab && m->embed->cols == c.hidden, N730_BAD_ARG,
               "model: embedding is %dx%d, expected %dx%d", m->embed->rows, m->embed->cols, c.vocab, c.hidden);
  m->lm_head = W(-1, N730_W_LMHEAD);
  if (!m->lm_head) {
    N730_REQUIRE(c.tie_embeddings, N730_STATE, "model: lm_head not set and embeddings not tied");
    m->lm_head = m->embed;
  }
  m->vocab_l = m->lm_head->rows;
  if (c.tp_size > 1) {
    N730_REQUIRE(m->comm, N730_STATE, "model: tensor parallel needs n730_model_tp_init before finalize");
    N730_REQUIRE(m->lm_head->rows == c.vocab || (long long)m->lm_head->rows * c.tp_size == c.vocab, N730_BAD_ARG,
                 "model: lm_head has %d rows: expected %d (replicated) or %d (vocab split)", m->lm_head->rows,
                 c.vocab, c.vocab / c.tp_size);
  } else {
    N730_REQUIRE(m->lm_head->rows == c.vocab && m->lm_head->cols == c.hidden, N730_BAD_ARG,
                 "model: lm_head is %dx%d, expected %dx%d", m->lm_head->rows, m->lm_head->cols, c.vocab, c.hidden);
  }
  m->qkv_dim = (c.heads + 2 * c.kv_heads) * c.head_dim;
  for (int l = 0; l < nl; ++l) {
    Layer& y = m->L[l];
    QWeight *q = W(l, N730_W_Q), *k = W(l, N730_W_K), *v = W(l, N730_W_V);
    N730_REQUIRE(q && k && v && W(l, N730_W_O) && W(l, N730_W_GATE) && W(l, N730_W_UP) && W(l, N730_W_DOWN),
                 N730_STATE, "model: layer %d is missing a projection", l);
    N730_REQUIRE(q->rows == c.heads * c.head_dim && k->rows == c.kv_heads * c.head_dim &&
                     v->rows == c.kv_heads * c.head_dim && q->cols == c.hidden,
                 N730_BAD_ARG, "model: layer %d q/k/v shapes do not match the config", l);
    if (int rc = fuse_rows(m, {q, k, v}, false, &y.qkv)) return rc;
    y.o = W(l, N730_W_O);
    if (int rc = fuse_rows(m, {W(l, N730_W_GATE), W(l, N730_W_UP)}, true, &y.gate_up)) return rc;
    y.down = W(l, N730_W_DOWN);
    N730_REQUIRE(y.o->rows == c.hidden && y.o->cols == c.heads * c.head_dim && y.gate_up->rows == 2 * c.ffn &&
                     y.gate_up->cols == c.hidden && y.down->rows == c.hidden && y.down->cols == c.ffn,
                 N730_BAD_ARG, "model: layer %d o/gate/up/down shapes do not match the config", l);
    std::vector<float> ones(c.hidden, 1.f);
    const std::vector<float>* n1 = V(l, N730_V_INPUT_NORM);
    const std::vector<float>* n2 = V(l, N730_V_POST_NORM);
    if (int rc = upload_vec(m, n1 ? *n1 : ones, &y.ln1)) return rc;
    if (int rc = upload_vec(m, n2 ? *n2 : ones, &y.ln2)) return rc;
    const auto *bq = V(l, N730_V_Q_BIAS), *bk = V(l, N730_V_K_BIAS), *bv = V(l, N730_V_V_BIAS);
    if (bq || bk || bv) {
      std::vector<float> b(m->qkv_dim, 0.f);
      if (bq) std::copy(bq->begin(), bq->end(), b.begin());
      if (bk) std::copy(bk->begin(), bk->end(), b.begin() + c.heads * c.head_dim);
      if (bv) std::copy(bv->begin(), bv->end(), b.begin() + (c.heads + c.kv_heads) * c.head_dim);
      if (int rc = upload_vec(m, b, &y.qkv_bias)) return rc;
    }
    if (const auto* bo = V(l, N730_V_O_BIAS))
      if (int rc = upload_vec(m, *bo, &y.o_bias)) return rc;
    if (const auto* bd = V(l, N730_V_DOWN_BIAS))
      if (int rc = upload_vec(m, *bd, &y.down_bias)) return rc;
    const auto *bg = V(l, N730_V_GATE_BIAS), *bu = V(l, N730_V_UP_BIAS);
    if (bg || bu) {
      std::vector<float> b(2 * c.ffn, 0.f);
      for (int i = 0; i < c.ffn; ++i) {
        if (bg) b[2 * i] = (*bg)[i];
        if (bu) b[2 * i + 1] = (*bu)[i];
      }
      if (int rc = upload_vec(m, b, &y.gate_up_bias)) return rc;
    }
  }
  {
    std::vector<float> ones(c.hidden, 1.f);
    const std::vector<float>* fn = V(-1, N730_V_FINAL_NORM);
    if (int rc = upload_vec(m, fn ? *fn : ones, &m->final_norm)) return rc;
  }
  N730_CUDA(cudaStreamSynchronize(m->st));
  if (!c.exact_gemv) {  // INT4 group-wise weights -> tensor-core fragment tiles
    auto conv = [&](QWeight* w) -> int {
      if (w && w->bits == 4 && w->sz_mode == 0 && w->group % 64 == 0 && w->cols % 64 == 0 && w->layout == 0)
        return qweight_to_mma_layout(*w, m->st);
      return N730_OK;
    };
    for (auto& y : m->L)
      for (QWeight* w : {y.qkv, y.o, y.gate_up, y.down})
        if (int rc = conv(w)) return rc;
    if (int rc = conv(m->embed)) return rc;
    if (m->lm_head != m->embed)
      if (int rc = conv(m->lm_head)) return rc;
  }
  if (c.stream_depth > 0)
    if (int rc = setup_streaming(m)) return rc;
  for (auto& kv : m->pend_w) {
    const int s = kv.first.second;
    if (s == N730_W_Q || s == N730_W_K || s == N730_W_V || s == N730_W_GATE || s == N730_W_UP)
      qweight_destroy(kv.second);
  }
  m->pend_w.clear();
  m->pend_v.clear();

  // RoPE tables as the reference builds them (n730_cuda.cu:650-661)
  const int h2 = c.head_dim / 2;
  {
    std::vector<float> hc((size_t)c.max_ctx * h2), hs((size_t)c.max_ctx * h2);
    for (int pos = 0; pos < c.max_ctx; ++pos)
      for (int i = 0; i < h2; ++i) {
        const float freq = 1.0f / powf(c.rope_theta, (float)(2 * i) / c.head_dim);
        const float ang = pos * freq;
        hc[(size_t)pos * h2 + i] = cosf(ang);
        hs[(size_t)pos * h2 + i] = sinf(ang);
      }
    if (int rc = upload_vec(m, hc, &m->cos_t)) return rc;
    if (int rc = upload_vec(m, hs, &m->sin_t)) return rc;
  }
  // paged KV: a pool of pages (max_batch x pages per sequence unless kv_pool_pages asks for fewer),
  // handed to sequences as they grow (ensure_pages) and returned when they are released
  m->max_pages = (c.max_ctx + c.page_size - 1) / c.page_size;
  const size_t table = (size_t)c.max_batch * m->max_pages;
  const size_t pages = c.kv_pool_pages > 0 ? std::min(table, (size_t)c.kv_pool_pages) : table;
  m->pool_pages = (int)pages;
  const size_t per_layer = pages * c.kv_heads * c.page_size * c.head_dim;
  if (int rc = m->alloc(&m->k_pool, per_layer * nl)) return rc;
  if (int rc = m->alloc(&m->v_pool, per_layer * nl)) return rc;
  N730_CUDA(cudaMemsetAsync(m->k_pool, 0, per_layer * nl * sizeof(__half), m->st));
  N730_CUDA(cudaMemsetAsync(m->v_pool, 0, per_layer * nl * sizeof(__half), m->st));
  for (int l = 0; l < nl; ++l) m->L[l].kv = KVLayer{m->k_pool + per_layer * l, m->v_pool + per_layer * l};
  {
    // unassigned entries point at page 0 (in bounds); kernels read entries below a sequence's length only
    m->h_bt.assign(table, 0);
    if (int rc = m->alloc(&m->block_table, table)) return rc;
    N730_CUDA(cudaMemcpyAsync(m->block_table, m->h_bt.data(), table * 4, cudaMemcpyHostToDevice, m->st));
    m->free_pages.resize(pages);
    for (size_t i = 0; i < pages; ++i) m->free_pages[i] = (int)(pages - 1 - i);  // page 0 handed out first
    m->seq_pages.assign(c.max_batch, {});
  }
  if (int rc = m->alloc(&m->seq_lens, c.max_batch)) return rc;
  N730_CUDA(cudaMemsetAsync(m->seq_lens, 0, c.max_batch * 4, m->st));
  m->h_seq.assign(c.max_batch, 0);
  // decode workspace
  const int B = c.max_batch;
  m->n_split = 8;  // context splits per (sequence, KV head): one 8-CTA cluster
  if (int rc = m->alloc(&m->d_tokens, B)) return rc;
  if (int rc = m->alloc(&m->x, (size_t)B * c.hidden)) return rc;
  if (int rc = m->alloc(&m->qkv, (size_t)B * m->qkv_dim)) return rc;
  if (int rc = m->alloc(&m->attn, (size_t)B * c.heads * c.head_dim)) return rc;
  if (int rc = m->alloc(&m->mlp, (size_t)B * c.ffn)) return rc;
  if (int rc = m->alloc(&m->logits, (size_t)B * c.vocab)) return rc;
  if (int rc = m->alloc(&m->rms_ws, (size_t)std::max(B, c.max_prefill))) return rc;
  if (int rc = m->alloc(&m->ss_ws, (size_t)std::max(B, c.max_prefill) * ((c.hidden + TC_SS_ROWS - 1) / TC_SS_ROWS)))
    return rc;
  if (B > 1) {  // split-K partials of batched GEMVs whose x does not fit shared memory (down_proj)
    m->split_ws_floats = (int64_t)16 * std::min(B, 16) * c.hidden;
    if (int rc = m->alloc(&m->split_ws, (size_t)m->split_ws_floats)) return rc;
  }
  if (c.tp_size > 1) {
    if (int rc = m->alloc(&m->delta, (size_t)std::max(B, c.max_prefill) * c.hidden)) return rc;
    if (m->vocab_l != c.vocab)
      if (int rc = m->alloc(&m->logits_all, (size_t)c.tp_size * B * m->vocab_l)) return rc;
  }
  // prefill workspace
  const int P = c.max_prefill;
  if (int rc = m->alloc(&m->p_tokens, P)) return rc;
  if (int rc = m->alloc(&m->px, (size_t)P * c.hidden)) return rc;
  if (int rc = m->alloc(&m->pqkv, (size_t)P * m->qkv_dim)) return rc;
  if (int rc = m->alloc(&m->pattn, (size_t)P * c.heads * c.head_dim)) return rc;
  if (int rc = m->alloc(&m->pmlp, (size_t)P * c.ffn)) return rc;
  N730_CUDA(cudaMallocHost(&m->h_tok, (size_t)std::max(B, P) * 4));
  N730_CUDA(cudaMallocHost(&m->h_logits, (size_t)B * c.vocab * 4));
  if (c.per_op_decode <= 0)
    if (int rc = plan_persistent(m)) return rc;
  if (c.tp_size > 1)
    if (int rc = agree_decode_path(m)) return rc;
  N730_CUDA(cudaStreamSynchronize(m->st));
  m->finalized = true;
  return N730_OK;
}

// GEMM or GEMV for `batch` rows.  From GEMM_TC_MIN_TOKENS rows on the tcgen05 GEMM
// (each weight dequantised once per token tile).  From 9 to 127 rows the GEMV streams
// the weights once per 16 rows with twice the tensor-core work of 8, so the GEMM
// (32- to 128-token tile, K split over CTAs for narrow linears) takes every linear whose
// grid (with the split) fills the SMs; measured on the 7B shape: gate|up at 32 rows 37 us
// against 126 us for the GEMV, decode steps of 16 sequences 4381 against 4202 tok/s with
// the narrow linears on the GEMV; at <= 8 rows the GEMV is faster (gate|up 27 us).
static bool use_gemm_tc(const QWeight& w, int batch, bool swiglu) {
  if (!gemm_tc_supported(w, batch)) return false;
  if (batch >= GEMM_TC_MIN_TOKENS) return true;
  if (batch <= 8) return false;
  return gemm_tc_ctas(w.rows, w.cols, batch, swiglu) >= num_sms();
}

// Rows from which the split-K fold hands sums of squares to the next RMSNorm.  Measured on
// the 7B shape, same box against the same build without the hand-off: 32 sequences 8008 ->
// 8328 tok/s, but 16 sequences 4582 -> 4204, so smaller batches keep the 1/rms kernel.
constexpr int SS_MIN_ROWS = 32;

// One linear for `batch` rows of x (use_gemm_tc picks the kernel).  `sums`: y is the
// residual stream; a split-K GEMM's fold then also leaves its sums of squares for the
// next RMSNorm'd GEMM of y (from SS_MIN_ROWS rows), which reads them instead of a pass over y.
static int gemv(Model* m, const QWeight* w, const float* x, int ldx, int batch, float* y, int ldy,
                const float* bias, const float* resid, int ldr, const float* norm, int swiglu, bool sums = false) {
  GemvArgs a = {};
  a.w = w; a.x = x; a.ldx = ldx; a.batch = batch; a.y = y; a.ldy = ldy; a.bias = bias;
  a.residual = resid; a.ldr = ldr; a.norm_w = norm; a.eps = m->c.rms_eps; a.swiglu = swiglu;
  a.pdl = m->c.use_pdl;
  if (w->rows <= m->c.hidden) { a.split_ws = m->split_ws; a.split_ws_floats = m->split_ws_floats; }
  const int h = m->c.hidden;
  const bool tc = use_gemm_tc(*w, batch, swiglu != 0) && !m->c.exact_gemv;
  if (tc && norm && m->ss_of == x && m->ss_rows == batch && ldx == h && w->cols == h) a.ss_in = m->ss_ws;
  m->ss_of = nullptr;
  const bool ss_out = tc && sums && batch >= SS_MIN_ROWS && w->rows == h && ldy == h && batch <= std::max(m->c.max_batch, m->c.max_prefill) &&
                      gemm_tc_folds(*w, batch, swiglu != 0);
  if (ss_out) a.ss_out = m->ss_ws;
  if (!tc) return gemv_launch(a, m->st);
  if (int rc = gemm_tc_launch(a, m->rms_ws, m->st)) return rc;
  if (ss_out) { m->ss_of = y; m->ss_rows = batch; }
  return N730_OK;
}

static int launch_add(Model* m, float* x, const float* d, int64_t n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms()));
  cfg.blockDim = dim3(256);
  cfg.stream = m->st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = m->c.use_pdl ? 1 : 0;
  N730_CUDA(cudaLaunchKernelEx(&cfg, add_inplace_kernel, x, d, n));
  return N730_OK;
}

// y = x_res + W a (+ bias): the row-split projections o_proj / down_proj.  With
// tensor parallelism W holds this rank's K columns: the partial products are
// summed across ranks by one allreduce, then added to the residual stream.
static int rowsplit_linear(Model* m, const QWeight* w, const float* a, int lda, int B, float* x, int ldx,
                           const float* bias) {
  if (m->c.tp_size <= 1) return gemv(m, w, a, lda, B, x, ldx, bias, x, ldx, nullptr, 0, true);
  const int h = m->c.hidden;
  if (int rc = gemv(m, w, a, lda, B, m->delta, h, bias, nullptr, 0, nullptr, 0)) return rc;
  if (m->ar_ok && !m->ar_off && m->c.tp_allreduce == 0 && (int64_t)B * h <= m->ar.cap && ldx == h) {  // one-shot
    ArArgs ar = m->ar;
    ar.part = m->delta;
    ar.x = x;
    ar.n = B * h;
    return ar_launch(ar, m->st);
  }
  if (ncclAllReduce(m->delta, m->delta, (size_t)B * h, ncclFloat, ncclSum, m->comm, m->st) != ncclSuccess) {
    set_error("model: ncclAllReduce failed");
    return N730_COMM;
  }
  N730_REQUIRE(ldx == h, N730_BAD_ARG, "model: residual stride");
  return launch_add(m, x, m->delta, (int64_t)B * h);
}

static int gather_logits(Model* m, int B, float* logits);

// logits [B][vocab] = lm_head(final_norm(x)); vocab-split lm_head: gather the shards
static int lm_head_logits(Model* m, const float* x, int B, float* logits) {
  const N730ModelConfig& c = m->c;
  if (m->vocab_l == c.vocab)
    return gemv(m, m->lm_head, x, c.hidden, B, logits, c.vocab, nullptr, nullptr, 0, m->final_norm, 0);
  float* part = m->logits_all + (size_t)c.tp_rank * B * m->vocab_l;
  if (int rc = gemv(m, m->lm_head, x, c.hidden, B, part, m->vocab_l, nullptr, nullptr, 0, m->final_norm, 0))
    return rc;
  return gather_logits(m, B, logits);
}

// vocab-split lm_head: every rank's shard (logits_all[rank]) -> logits [B][vocab]
static int gather_logits(Model* m, int B, float* logits) {
  const N730ModelConfig& c = m->c;
  float* part = m->logits_all + (size_t)c.tp_rank * B * m->vocab_l;
  if (ncclAllGather(part, m->logits_all, (size_t)B * m->vocab_l, ncclFloat, m->comm, m->st) != ncclSuccess) {
    set_error("model: ncclAllGather failed");
    return N730_COMM;
  }
  const int64_t n = (int64_t)c.tp_size * B * m->vocab_l;
  gather_logits_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4 * num_sms()), 256, 0, m->st>>>(
      m->logits_all, logits, c.tp_size, B, m->vocab_l);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

static AttnDims dims(const Model* m) {
  AttnDims d{};
  d.n_heads = m->c.heads; d.n_kv = m->c.kv_heads; d.head_dim = m->c.head_dim;
  d.page_size = m->c.page_size; d.max_pages = m->max_pages;
  d.scale = 1.0f / sqrtf((float)m->c.head_dim);
  return d;
}

// Enqueue one decode step for sequences [0, B) on m->st (tokens in m->d_tokens).
static int enqueue_decode(Model* m, int B) {
  const N730ModelConfig& c = m->c;
  const int h = c.hidden, ad = c.heads * c.head_dim;
  m->ss_of = nullptr;  // x is rewritten by the embedding
  if (int rc = embed_launch(*m->embed, m->d_tokens, B, m->x, m->st)) return rc;
  const bool persistent = B == 1 && m->pd_ok;
  if (persistent) {
    if (int rc = persist_launch(m->pd, m->st)) return rc;
    if (c.tp_size > 1 && m->vocab_l != c.vocab)  // the kernel wrote this rank's vocab shard
      if (int rc = gather_logits(m, 1, m->logits)) return rc;
  }
  if (!persistent)
    if (int rc = stream_begin(m)) return rc;
  for (int l = 0; l < c.layers && !persistent; ++l) {
    Layer& y = m->L[l];
    LayerW lw;
    if (int rc = stream_acquire(m, l, &lw)) return rc;
    if (int rc = gemv(m, lw.qkv, m->x, h, B, m->qkv, m->qkv_dim, y.qkv_bias, nullptr, 0, y.ln1, 0)) return rc;
    DecodeAttnArgs a = {};
    a.qkv = m->qkv; a.ld_qkv = m->qkv_dim; a.cos_t = m->cos_t; a.sin_t = m->sin_t;
    a.seq_lens = m->seq_lens; a.block_table = m->block_table; a.kv = y.kv; a.d = dims(m);
    a.out = m->attn; a.batch = B; a.pdl = c.use_pdl;
    if (int rc = attn_decode_launch(a, m->st)) return rc;
    if (int rc = rowsplit_linear(m, lw.o, m->attn, ad, B, m->x, h, y.o_bias)) return rc;
    if (int rc = gemv(m, lw.gate_up, m->x, h, B, m->mlp, c.ffn, y.gate_up_bias, nullptr, 0, y.ln2, 1)) return rc;
    if (int rc = rowsplit_linear(m, lw.down, m->mlp, c.ffn, B, m->x, h, y.down_bias)) return rc;
    if (int rc = stream_release(m, l)) return rc;
  }
  if (!persistent)
    if (int rc = lm_head_logits(m, m->x, B, m->logits)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((B + 127) / 128);
  cfg.blockDim = dim3(128);
  cfg.stream = m->st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = c.use_pdl ? 1 : 0;
  N730_CUDA(cudaLaunchKernelEx(&cfg, advance_seq_kernel, m->seq_lens, B, 1));
  return N730_OK;
}

static int run_decode(Model* m, int B) {
  if (!m->c.use_graphs || m->c.stream_depth > 0) return enqueue_decode(m, B);
  auto it = m->graphs.find(B);
  if (it == m->graphs.end()) {
    cudaGraph_t g = nullptr;
    N730_CUDA(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_decode(m, B);
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    N730_CUDA(e);
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    N730_CUDA(e);
    it = m->graphs.emplace(B, ex).first;
  }
  N730_CUDA(cudaGraphLaunch(it->second, m->st));
  return N730_OK;
}

// Give sequence b pages for positions [0, len) from the pool and upload its new block-table
// entries (asynchronously on the model stream, ahead of the kernels that read them).
static int ensure_pages(Model* m, int b, int len) {
  const int need = (len + m->c.page_size - 1) / m->c.page_size;
  std::vector<int>& own = m->seq_pages[b];
  const int have = (int)own.size();
  if (need <= have) return N730_OK;
  N730_REQUIRE(need - have <= (int)m->free_pages.size(), N730_STATE,
               "KV page pool exhausted: sequence %d needs %d more pages, %zu free of %d", b, need - have,
               m->free_pages.size(), m->pool_pages);
  for (int k = have; k < need; ++k) {
    own.push_back(m->free_pages.back());
    m->free_pages.pop_back();
    m->h_bt[(size_t)b * m->max_pages + k] = own.back();
  }
  const size_t o = (size_t)b * m->max_pages + have;
  N730_CUDA(cudaMemcpyAsync(m->block_table + o, m->h_bt.data() + o, (size_t)(need - have) * 4, cudaMemcpyHostToDevice,
                            m->st));
  return N730_OK;
}

static int check_capacity(Model* m, int b, int add) {
  N730_REQUIRE(m->h_seq[b] + add <= m->c.max_ctx, N730_STATE,
               "KV cache capacity exceeded: %d tokens requested, maximum is %d", m->h_seq[b] + add, m->c.max_ctx);
  if (int rc = ensure_pages(m, b, m->h_seq[b] + add)) return rc;
  return N730_OK;
}

static int prefill(Model* m, int seq, const int32_t* d_tok, int T, float* d_logits_row) {
  const N730ModelConfig& c = m->c;
  const int h = c.hidden, ad = c.heads * c.head_dim;
  int done = 0;
  while (done < T) {
    const int n = std::min(c.max_prefill, T - done);
    const int pos0 = m->h_seq[seq] + done;
    m->ss_of = nullptr;  // px is rewritten by the embedding
    if (int rc = embed_launch(*m->embed, d_tok + done, n, m->px, m->st)) return rc;
    if (int rc = stream_begin(m)) return rc;
    for (int l = 0; l < c.layers; ++l) {
      Layer& y = m->L[l];
      LayerW lw;
      if (int rc = stream_acquire(m, l, &lw)) return rc;
      if (int rc = gemv(m, lw.qkv, m->px, h, n, m->pqkv, m->qkv_dim, y.qkv_bias, nullptr, 0, y.ln1, 0)) return rc;
      KVWriteArgs kw = {};
      kw.qkv = m->pqkv; kw.ld_qkv = m->qkv_dim; kw.cos_t = m->cos_t; kw.sin_t = m->sin_t;
      kw.block_table = m->block_table + (size_t)seq * m->max_pages; kw.kv = y.kv; kw.d = dims(m);
      kw.T = n; kw.pos0 = pos0; kw.pdl = c.use_pdl;
      if (int rc = kv_write_launch(kw, m->st)) return rc;
      PrefillAttnArgs pa = {};
      pa.qkv = m->pqkv; pa.ld_qkv = m->qkv_dim; pa.block_table = kw.block_table; pa.kv = y.kv; pa.d = dims(m);
      pa.T = n; pa.pos0 = pos0; pa.out = m->pattn; pa.pdl = c.use_pdl;
      if (int rc = attn_prefill_launch(pa, m->st)) return rc;
      if (int rc = rowsplit_linear(m, lw.o, m->pattn, ad, n, m->px, h, y.o_bias)) return rc;
      if (int rc = gemv(m, lw.gate_up, m->px, h, n, m->pmlp, c.ffn, y.gate_up_bias, nullptr, 0, y.ln2, 1)) return rc;
      if (int rc = rowsplit_linear(m, lw.down, m->pmlp, c.ffn, n, m->px, h, y.down_bias)) return rc;
      if (int rc = stream_release(m, l)) return rc;
    }
    done += n;
    if (done == T && d_logits_row)
      if (int rc = lm_head_logits(m, m->px + (size_t)(n - 1) * h, 1, d_logits_row)) return rc;
  }
  return N730_OK;
}

}  // namespace n730

using namespace n730;

#define MODEL(p) Model* m = (Model*)(p); if (!m) return N730_NULL

N730_API int n730_model_create(const N730ModelConfig* cfg, void** out) {
  if (!cfg || !out) return N730_NULL;
  *out = nullptr;
  const N730ModelConfig& c = *cfg;
  N730_REQUIRE(c.hidden > 0 && c.layers > 0 && c.heads > 0 && c.kv_heads > 0 && c.heads % c.kv_heads == 0 &&
                   c.head_dim > 0 && c.ffn > 0 && c.vocab > 0 && c.max_ctx > 0 && c.max_batch > 0,
               N730_BAD_ARG, "model_create: invalid config");
  N730_REQUIRE(c.head_dim == 64 || c.head_dim == 128, N730_UNSUPPORTED, "model_create: head_dim %d", c.head_dim);
  N730_REQUIRE(c.stream_depth >= 0 && c.stream_depth <= 16, N730_BAD_ARG, "model_create: stream_depth %d",
               c.stream_depth);
  Model* m = new Model();
  m->c = c;
  if (m->c.page_size <= 0) m->c.page_size = 64;
  if (m->c.max_prefill <= 0) m->c.max_prefill = 512;
  if (m->c.tp_size <= 0) m->c.tp_size = 1;
  cudaGetDevice(&m->device);
  if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
    delete m;
    return N730_CUDA_ERR;
  }
  *out = m;
  return N730_OK;
}

N730_API int n730_tp_unique_id(uint8_t* out) {
  if (!out) return N730_NULL;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) {
    set_error("ncclGetUniqueId failed");
    return N730_COMM;
  }
  memcpy(out, &id, sizeof id);
  return N730_OK;
}

N730_API int n730_model_tp_init(void* p, const uint8_t* id_bytes, int rank, int size) {
  MODEL(p);
  N730_REQUIRE(id_bytes, N730_NULL, "tp_init: null id");
  N730_REQUIRE(!m->finalized && !m->comm, N730_STATE, "tp_init: call once, before finalize");
  N730_REQUIRE(size == m->c.tp_size && rank == m->c.tp_rank && size > 1, N730_BAD_ARG,
               "tp_init: rank %d of %d does not match the config (%d of %d)", rank, size, m->c.tp_rank,
               m->c.tp_size);
  ncclUniqueId id;
  memcpy(&id, id_bytes, sizeof id);
  N730_CUDA(cudaSetDevice(m->device));
  if (ncclCommInitRank(&m->comm, size, id, rank) != ncclSuccess) {
    m->comm = nullptr;
    set_error("ncclCommInitRank failed (rank %d of %d)", rank, size);
    return N730_COMM;
  }
  if (size <= AR_MAX_RANKS) {  // exchange region: one-shot allreduce, persistent decode's exchanges
    const int64_t cap = ((int64_t)m->c.max_batch * m->c.hidden + 3) / 4 * 4;
    N730_CUDA(cudaMalloc(&m->ar_base, ar_region_bytes(size, cap)));
    N730_CUDA(cudaMemset(m->ar_base, 0, ar_region_bytes(size, cap)));
    int* ctr = nullptr;
    if (int rc = m->alloc(&ctr, 2)) return rc;
    N730_CUDA(cudaMemset(ctr, 0, 8));
    N730_CUDA(cudaDeviceSynchronize());
    m->ar.rank = rank;
    m->ar.size = size;
    m->ar.cap = cap;
    m->ar.local = ar_region_at(m->ar_base, size);
    m->ar.peer[rank] = m->ar.local;
    m->ar.epoch = ctr;
    m->ar.done = ctr + 1;
    m->ar.err = gemv_err_word();
    N730_REQUIRE(m->ar.err, N730_OOM, "tp_init: error word allocation failed");
  }
  return N730_OK;
}

N730_API int n730_model_tp_ipc_handle(void* p, uint8_t* out) {
  MODEL(p);
  N730_REQUIRE(out, N730_NULL, "tp_ipc_handle: null output");
  N730_REQUIRE(m->ar_base, N730_STATE, "tp_ipc_handle: no exchange region (tp_init first, at most %d ranks)",
               AR_MAX_RANKS);
  cudaIpcMemHandle_t hd;
  N730_CUDA(cudaIpcGetMemHandle(&hd, m->ar_base));
  static_assert(sizeof(cudaIpcMemHandle_t) == N730_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(out, &hd, sizeof hd);
  return N730_OK;
}

N730_API int n730_model_tp_ipc_open(void* p, const uint8_t* handles, int size) {
  MODEL(p);
  N730_REQUIRE(handles, N730_NULL, "tp_ipc_open: null handles");
  N730_REQUIRE(m->ar_base && size == m->ar.size && !m->ar_ok, N730_STATE,
               "tp_ipc_open: once, after tp_ipc_handle, with every rank's handle");
  N730_CUDA(cudaSetDevice(m->device));
  for (int r = 0; r < size; ++r) {
    if (r == m->ar.rank) continue;
    cudaIpcMemHandle_t hd;
    memcpy(&hd, handles + (size_t)r * sizeof hd, sizeof hd);
    void* ptr = nullptr;
    N730_CUDA(cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess));
    m->ar_peer_base.push_back(ptr);
    m->ar.peer[r] = ar_region_at(ptr, size);
  }
  m->ar_ok = true;
  return N730_OK;
}

N730_API void n730_model_destroy(void* p) {
  Model* m = (Model*)p;
  if (!m) return;
  cudaStreamSynchronize(m->st);
  for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);  // graphs holding NCCL calls go before the comm
  for (void* q : m->ar_peer_base) cudaIpcCloseMemHandle(q);
  if (m->ar_base) cudaFree(m->ar_base);
  if (m->comm) ncclCommDestroy(m->comm);
  for (auto& kv : m->pend_w) qweight_destroy(kv.second);
  for (auto& y : m->L) {
    qweight_destroy(y.qkv); qweight_destroy(y.o); qweight_destroy(y.gate_up); qweight_destroy(y.down);
  }
  if (m->lm_head != m->embed) qweight_destroy(m->lm_head);
  qweight_destroy(m->embed);
  for (void* a : m->allocs) cudaFree(a);
  for (uint8_t* im : m->img) if (im) cudaFreeHost(im);
  for (auto e : m->ev_ready) if (e) cudaEventDestroy(e);
  for (auto e : m->ev_free) if (e) cudaEventDestroy(e);
  if (m->cst) cudaStreamDestroy(m->cst);
  if (m->h_tok) cudaFreeHost(m->h_tok);
  if (m->h_logits) cudaFreeHost(m->h_logits);
  cudaStreamDestroy(m->st);
  delete m;
}

N730_API int n730_model_set_qweight(void* p, int layer, int slot, void* qw) {
  MODEL(p);
  N730_REQUIRE(!m->finalized, N730_STATE, "model: already finalized");
  N730_REQUIRE(qw, N730_NULL, "model: null weight");
  const bool global = slot == N730_W_EMBED || slot == N730_W_LMHEAD;
  N730_REQUIRE(global ? layer == -1 : (layer >= 0 && layer < m->c.layers && slot >= N730_W_Q && slot <= N730_W_DOWN),
               N730_BAD_ARG, "model: bad weight slot %d for layer %d", slot, layer);
  auto key = std::make_pair(layer, slot);
  auto it = m->pend_w.find(key);
  if (it != m->pend_w.end()) qweight_destroy(it->second);
  m->pend_w[key] = (QWeight*)qw;
  return N730_OK;
}

N730_API int n730_model_set_vector(void* p, int layer, int slot, const float* data, int n, int on_device) {
  MODEL(p);
  N730_REQUIRE(!m->finalized, N730_STATE, "model: already finalized");
  N730_REQUIRE(data && n > 0, N730_NULL, "model: null vector");
  std::vector<float> v(n);
  if (on_device) N730_CUDA(cudaMemcpy(v.data(), data, (size_t)n * 4, cudaMemcpyDeviceToHost));
  else memcpy(v.data(), data, (size_t)n * 4);
  m->pend_v[{layer, slot}] = std::move(v);
  return N730_OK;
}

N730_API int n730_model_finalize(void* p) {
  MODEL(p);
  N730_REQUIRE(!m->finalized, N730_STATE, "model: already finalized");
  return finalize(m);
}

// Return sequence b's pages to the pool (its length becomes 0).
static void release_pages(Model* m, int b) {
  for (int k = (int)m->seq_pages[b].size() - 1; k >= 0; --k) m->free_pages.push_back(m->seq_pages[b][k]);
  m->seq_pages[b].clear();
}

N730_API int n730_model_reset(void* p) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_CUDA(cudaStreamSynchronize(m->st));
  for (int b = 0; b < m->c.max_batch; ++b) release_pages(m, b);
  std::fill(m->h_seq.begin(), m->h_seq.end(), 0);
  N730_CUDA(cudaMemsetAsync(m->seq_lens, 0, m->c.max_batch * 4, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  return N730_OK;
}

// Set a sequence's cached length (positions [0, len) are taken as already in
// the KV cache).  Used to resume a sequence whose cache was filled earlier
// and to position decode benchmarks at a given context.
N730_API int n730_model_set_seq_len(void* p, int seq, int len) {
  MODEL(p);
  N730_REQUIRE(m->finalized && seq >= 0 && seq < m->c.max_batch && len >= 0 && len <= m->c.max_ctx,
               N730_BAD_ARG, "set_seq_len: bad sequence %d or length %d", seq, len);
  if (int rc = ensure_pages(m, seq, len)) return rc;
  m->h_seq[seq] = len;
  N730_CUDA(cudaMemcpyAsync(m->seq_lens + seq, &m->h_seq[seq], 4, cudaMemcpyHostToDevice, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  return N730_OK;
}

// Release sequence `seq`: its pages go back to the pool and its length becomes 0.
N730_API int n730_model_seq_release(void* p, int seq) {
  MODEL(p);
  N730_REQUIRE(m->finalized && seq >= 0 && seq < m->c.max_batch, N730_BAD_ARG, "seq_release: bad sequence %d", seq);
  N730_CUDA(cudaStreamSynchronize(m->st));  // no kernel of an earlier step still reads its pages
  release_pages(m, seq);
  m->h_seq[seq] = 0;
  N730_CUDA(cudaMemcpyAsync(m->seq_lens + seq, &m->h_seq[seq], 4, cudaMemcpyHostToDevice, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  return N730_OK;
}

// Move sequence `src` (pages, block-table row, length) into the empty slot `dst`; src becomes empty.
// Decode steps run sequences [0, batch), so a batch is compacted by moving its last sequence into
// the slot of one that finished: no KV data moves, only the row of page ids.
N730_API int n730_model_seq_move(void* p, int dst, int src) {
  MODEL(p);
  const int B = m->c.max_batch;
  N730_REQUIRE(m->finalized && dst >= 0 && dst < B && src >= 0 && src < B && dst != src, N730_BAD_ARG,
               "seq_move: bad slots %d <- %d", dst, src);
  N730_REQUIRE(m->seq_pages[dst].empty() && m->h_seq[dst] == 0, N730_STATE, "seq_move: slot %d is not empty", dst);
  N730_CUDA(cudaStreamSynchronize(m->st));
  m->seq_pages[dst].swap(m->seq_pages[src]);
  const size_t P = m->max_pages;
  for (size_t k = 0; k < P; ++k) m->h_bt[dst * P + k] = m->h_bt[src * P + k];
  m->h_seq[dst] = m->h_seq[src];
  m->h_seq[src] = 0;
  N730_CUDA(cudaMemcpyAsync(m->block_table + dst * P, m->h_bt.data() + dst * P, P * 4, cudaMemcpyHostToDevice, m->st));
  N730_CUDA(cudaMemcpyAsync(m->seq_lens + dst, &m->h_seq[dst], 4, cudaMemcpyHostToDevice, m->st));
  N730_CUDA(cudaMemcpyAsync(m->seq_lens + src, &m->h_seq[src], 4, cudaMemcpyHostToDevice, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  return N730_OK;
}

// KV page pool: *free_pages and *total_pages (pages of page_size positions).
N730_API int n730_model_kv_pages(void* p, int* free_pages, int* total_pages) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  if (free_pages) *free_pages = (int)m->free_pages.size();
  if (total_pages) *total_pages = m->pool_pages;
  return N730_OK;
}

N730_API int n730_model_seq_len(void* p, int seq) {
  MODEL(p);
  N730_REQUIRE(seq >= 0 && seq < m->c.max_batch && m->finalized, N730_BAD_ARG, "model: bad sequence %d", seq);
  return m->h_seq[seq];
}

// Status of the work enqueued so far (call after a synchronisation).  A
// bounded device wait that ran out during a tensor-parallel step leaves the
// ranks' exchange counters (persistent kernel) or epochs (one-shot allreduce)
// out of step, so every later exchange over peer memory would wait for
// arrivals that never match.  After such a timeout the model stops using
// both for good: the persistent kernel and the one-shot allreduce are switched
// off and the captured step graphs dropped; later steps run the per-op kernels
// with NCCL.  The caller still gets N730_TIMEOUT for the failed step.
static int step_status(Model* m) {
  const int rc = gemv_check_error(true);
  if (rc == N730_TIMEOUT && m->c.tp_size > 1 && (m->pd_ok || (m->ar_ok && !m->ar_off))) {
    m->pd_ok = false;
    m->ar_off = true;
    for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
    m->graphs.clear();
  }
  return rc;
}

// Decode one token for each of sequences [0, batch): host token ids in,
// host logits [batch][vocab] out (pinned staging, copies inside the call).
static bool is_pinned_host(const void* ptr) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
    cudaGetLastError();  // clear the error this query leaves behind
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

// Page-locked host memory (e.g. the logits buffer a caller reuses across
// n730_model_decode calls: the copy then lands in it directly).
N730_API int n730_host_alloc(size_t bytes, void** out) {
  N730_REQUIRE(out && bytes > 0, N730_BAD_ARG, "host_alloc: %zu bytes", bytes);
  *out = nullptr;
  N730_CUDA(cudaMallocHost(out, bytes));
  return N730_OK;
}

N730_API int n730_host_free(void* ptr) {
  if (ptr) N730_CUDA(cudaFreeHost(ptr));
  return N730_OK;
}

N730_API int n730_model_decode(void* p, const int32_t* host_tokens, int batch, float* host_logits) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(host_tokens && batch >= 1 && batch <= m->c.max_batch, N730_BAD_ARG, "decode: batch %d", batch);
  for (int b = 0; b < batch; ++b) {
    N730_REQUIRE(host_tokens[b] >= 0 && host_tokens[b] < m->c.vocab, N730_BAD_ARG, "decode: token id %d out of range",
                 host_tokens[b]);
    if (int rc = check_capacity(m, b, 1)) return rc;
  }
  memcpy(m->h_tok, host_tokens, (size_t)batch * 4);
  N730_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tok, (size_t)batch * 4, cudaMemcpyHostToDevice, m->st));
  if (int rc = run_decode(m, batch)) return rc;
  // page-locked caller memory (n730_host_alloc, cudaHostRegister) takes the logits directly;
  // pageable memory gets them through the engine's pinned staging buffer
  const bool direct = host_logits && is_pinned_host(host_logits);
  if (host_logits) {
    N730_CUDA(cudaMemcpyAsync(direct ? host_logits : m->h_logits, m->logits, (size_t)batch * m->c.vocab * 4,
                              cudaMemcpyDeviceToHost, m->st));
  }
  N730_CUDA(cudaStreamSynchronize(m->st));
  if (host_logits && !direct) memcpy(host_logits, m->h_logits, (size_t)batch * m->c.vocab * 4);
  for (int b = 0; b < batch; ++b) m->h_seq[b] += 1;
  return step_status(m);
}

namespace n730 {
int sample_launch(const float* d_logits, int batch, int vocab, int ld, float temp, float top_p,
                  unsigned long long seed, unsigned long long counter, int32_t* d_tokens, float* d_u,
                  cudaStream_t st);
}

// Decode one token for each of sequences [0, batch) and sample the next tokens
// on the GPU (temperature + top-p, or greedy): host ids in, host ids out.
N730_API int n730_model_decode_sample(void* p, const int32_t* host_tokens, int batch, float temperature,
                                      float top_p, uint64_t seed, int32_t* host_next, float* host_u) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(host_tokens && host_next && batch >= 1 && batch <= m->c.max_batch, N730_BAD_ARG,
               "decode_sample: batch %d", batch);
  for (int b = 0; b < batch; ++b) {
    N730_REQUIRE(host_tokens[b] >= 0 && host_tokens[b] < m->c.vocab, N730_BAD_ARG, "decode: token id %d out of range",
                 host_tokens[b]);
    if (int rc = check_capacity(m, b, 1)) return rc;
  }
  if (!m->d_next) {
    if (int rc = m->alloc(&m->d_next, (size_t)2 * m->c.max_batch)) return rc;
  }
  memcpy(m->h_tok, host_tokens, (size_t)batch * 4);
  N730_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tok, (size_t)batch * 4, cudaMemcpyHostToDevice, m->st));
  if (int rc = run_decode(m, batch)) return rc;
  float* d_u = reinterpret_cast<float*>(m->d_next + m->c.max_batch);
  if (int rc = sample_launch(m->logits, batch, m->c.vocab, m->c.vocab, temperature, top_p, seed, m->sample_steps,
                             m->d_next, d_u, m->st))
    return rc;
  // tokens and u to the pinned staging buffer (the logits staging is large enough)
  N730_CUDA(cudaMemcpyAsync(m->h_logits, m->d_next, (size_t)batch * 4, cudaMemcpyDeviceToHost, m->st));
  N730_CUDA(cudaMemcpyAsync(m->h_logits + batch, d_u, (size_t)batch * 4, cudaMemcpyDeviceToHost, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  memcpy(host_next, m->h_logits, (size_t)batch * 4);
  if (host_u) memcpy(host_u, m->h_logits + batch, (size_t)batch * 4);
  for (int b = 0; b < batch; ++b) m->h_seq[b] += 1;
  ++m->sample_steps;
  return step_status(m);
}

// Device-resident decode step (no host copies, no synchronisation): d_tokens
// [batch] int32 and d_logits [batch][vocab] live in device memory; runs on
// `stream` after the model's own stream work.  Used to time the device path.
N730_API int n730_model_decode_device(void* p, const int32_t* d_tokens, int batch, float* d_logits, void* stream) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(batch >= 1 && batch <= m->c.max_batch, N730_BAD_ARG, "decode: batch %d", batch);
  for (int b = 0; b < batch; ++b) if (int rc = check_capacity(m, b, 1)) return rc;
  cudaStream_t us = (cudaStream_t)stream;
  cudaEvent_t ev;
  N730_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  if (us) { N730_CUDA(cudaEventRecord(ev, us)); N730_CUDA(cudaStreamWaitEvent(m->st, ev, 0)); }
  if (d_tokens) N730_CUDA(cudaMemcpyAsync(m->d_tokens, d_tokens, (size_t)batch * 4, cudaMemcpyDeviceToDevice, m->st));
  int rc = run_decode(m, batch);
  if (!rc && d_logits)
    rc = cuda_rc(cudaMemcpyAsync(d_logits, m->logits, (size_t)batch * m->c.vocab * 4, cudaMemcpyDeviceToDevice, m->st),
                 __FILE__, __LINE__);
  if (us) { cudaEventRecord(ev, m->st); cudaStreamWaitEvent(us, ev, 0); }
  cudaEventDestroy(ev);
  if (rc) return rc;
  for (int b = 0; b < batch; ++b) m->h_seq[b] += 1;
  return N730_OK;
}

// Launch only the persistent decode kernel of a batch-1 step on `stream` (the
// embedding and the position update are not run, so repeated calls recompute
// the same position).  Used to time that kernel alone.
N730_API int n730_model_run_step_kernel(void* p, void* stream) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(m->pd_ok, N730_UNSUPPORTED, "model: batch-1 decode does not use the persistent kernel");
  N730_REQUIRE(m->h_seq[0] < m->c.max_ctx, N730_STATE, "KV cache capacity exceeded");
  if (int rc = ensure_pages(m, 0, m->h_seq[0] + 1)) return rc;  // the step writes position h_seq[0]
  return persist_launch(m->pd, stream ? (cudaStream_t)stream : m->st);
}

// Run the persistent decode kernel of a batch-1 step once with per-phase
// timing (like n730_model_run_step_kernel: the position does not advance).
// host_times [6 n_phases + 1][grid] receives per CTA (%globaltimer ns): row 6p
// its arrival at the barrier before phase p (p = 0: the launch start), row
// 6p+1 its departure from that barrier, rows 6p+2 / 6p+3 marks inside the
// phase (GEMV: prologue done; FFN: prologue done, gate|up done; attention:
// split partial written, all splits of the head published; 0 where absent),
// rows 6p+4 / 6p+5 the time its warps spent waiting for weight chunks, summed
// over the warps (GEMV or gate|up; down_proj), the last row the end of its
// last phase; host_kinds [n_phases] the phase kinds (0 GEMV, 1 attention, 2 FFN).
// With host_times null only *n_phases and *grid are written (a size query).
N730_API int n730_model_trace_step(void* p, void* stream, uint64_t* host_times, int64_t cap, int8_t* host_kinds,
                                   int* n_phases, int* grid) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(m->pd_ok, N730_UNSUPPORTED, "model: batch-1 decode does not use the persistent kernel");
  N730_REQUIRE(m->h_seq[0] < m->c.max_ctx, N730_STATE, "KV cache capacity exceeded");
  if (int rc = ensure_pages(m, 0, m->h_seq[0] + 1)) return rc;  // the step writes position h_seq[0]
  const int np = m->pd.a.n_phases, g = m->pd.grid;
  if (n_phases) *n_phases = np;
  if (grid) *grid = g;
  if (!host_times) return N730_OK;
  const int64_t need = (int64_t)(PD_TRACE_ROWS * np + 1) * g;
  N730_REQUIRE(cap >= need, N730_BAD_ARG, "trace_step: %lld entries needed", (long long)need);
  if (!m->pd_trace)
    if (int rc = m->alloc(&m->pd_trace, (size_t)need)) return rc;
  cudaStream_t st = stream ? (cudaStream_t)stream : m->st;
  N730_CUDA(cudaMemsetAsync(m->pd_trace, 0, (size_t)need * 8, st));
  PdPlan plan = m->pd;
  plan.a.trace = m->pd_trace;
  if (int rc = persist_launch(plan, st)) return rc;
  N730_CUDA(cudaMemcpyAsync(host_times, m->pd_trace, (size_t)need * 8, cudaMemcpyDeviceToHost, st));
  N730_CUDA(cudaStreamSynchronize(st));
  if (host_kinds) memcpy(host_kinds, m->pd_kinds.data(), (size_t)np);
  return gemv_check_error(true);
}

// Append `n` tokens to sequence `seq` (prefill when n > 1, the decode graph
// when n == 1 and seq == 0) and return the logits of the last position.
N730_API int n730_model_forward(void* p, int seq, const int32_t* host_tokens, int n, float* host_logits) {
  MODEL(p);
  N730_REQUIRE(m->finalized, N730_STATE, "model: not finalized");
  N730_REQUIRE(host_tokens && n >= 1, N730_BAD_ARG, "forward requires at least one token");
  N730_REQUIRE(seq >= 0 && seq < m->c.max_batch, N730_BAD_ARG, "forward: bad sequence %d", seq);
  for (int i = 0; i < n; ++i)
    N730_REQUIRE(host_tokens[i] >= 0 && host_tokens[i] < m->c.vocab, N730_BAD_ARG, "token id %d out of range",
                 host_tokens[i]);
  if (int rc = check_capacity(m, seq, n)) return rc;
  if (n == 1 && seq == 0) return n730_model_decode(p, host_tokens, 1, host_logits);
  int done = 0;
  while (done < n) {  // chunks of the pinned staging size
    const int k = std::min(n - done, m->c.max_prefill);
    memcpy(m->h_tok, host_tokens + done, (size_t)k * 4);
    N730_CUDA(cudaMemcpyAsync(m->p_tokens, m->h_tok, (size_t)k * 4, cudaMemcpyHostToDevice, m->st));
    if (int rc = prefill(m, seq, m->p_tokens, k, done + k == n ? m->logits : nullptr)) return rc;
    N730_CUDA(cudaStreamSynchronize(m->st));
    m->h_seq[seq] += k;
    // the device copy of the length was written before this chunk's update
    N730_CUDA(cudaMemcpyAsync(m->seq_lens + seq, &m->h_seq[seq], 4, cudaMemcpyHostToDevice, m->st));
    done += k;
  }
  if (host_logits) N730_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToHost, m->st));
  N730_CUDA(cudaStreamSynchronize(m->st));
  if (host_logits) memcpy(host_logits, m->h_logits, (size_t)m->c.vocab * 4);
  return step_status(m);
}

// info[16]: weight bytes, kv bytes per position, kv capacity bytes, n_split,
// qkv_dim, max_pages, finalized, persistent batch-1 decode, untied embedding bytes,
// streamed layer bytes per pass, FFN fused, phase table in global memory,
// tensor-parallel plan mismatch, persistent grid
N730_API int n730_model_info(void* p, int64_t* info) {
  MODEL(p);
  if (!info) return N730_NULL;
  memset(info, 0, 16 * sizeof(int64_t));
  if (!m->finalized) return N730_OK;
  auto bytes = [](const QWeight* w) -> int64_t {
    if (!w) return 0;
    if (w->layout == 1) return (int64_t)((w->rows + 15) / 16) * w->n_groups * ((int64_t)(w->group / 16) * 128 + 64);
    return w->rows * w->row_bytes + (w->bits == 16 ? 0 : (int64_t)w->rows * w->sz_pitch);
  };
  int64_t wb = bytes(m->embed) + (m->lm_head != m->embed ? bytes(m->lm_head) : 0);
  for (auto& y : m->L) wb += bytes(y.qkv) + bytes(y.o) + bytes(y.gate_up) + bytes(y.down);
  info[0] = wb;
  info[1] = (int64_t)m->c.layers * 2 * m->c.kv_heads * m->c.head_dim * 2;
  info[2] = info[1] * (int64_t)m->pool_pages * m->c.page_size;
  info[3] = m->n_split;
  info[4] = m->qkv_dim;
  info[5] = m->max_pages;
  info[6] = m->finalized;
  info[7] = m->pd_ok;
  info[8] = m->lm_head != m->embed ? bytes(m->embed) : 0;  // read one row per token, not streamed
  info[9] = m->streamed_bytes;                                // host->HBM bytes per forward pass
  info[10] = m->pd_ffn_fused;
  info[11] = m->pd_ok && m->pd.a.tab_off < 0;  // persistent kernel reads its phase table from global memory
  info[12] = m->plan_mismatch;                 // tensor parallel: plans differed, every rank runs per-op
  info[13] = m->pd_ok ? m->pd.grid : 0;        // CTAs of the persistent launch
  return N730_OK;
}

N730_API void* n730_model_stream(void* p) { return p ? ((Model*)p)->st : nullptr; }

// Run one resident linear of the model alone (no norm / bias / residual):
// which = 0 q|k|v, 1 o_proj, 2 gate|up (SwiGLU), 3 down_proj, 4 lm_head.
// d_x [batch][cols], d_y [batch][rows] (rows/2 for gate|up).  Used to time
// the dequant-GEMV kernel on the model's real weights.
N730_API int n730_model_run_linear(void* p, int layer, int which, const float* d_x, int batch, float* d_y,
                                   void* stream) {
  MODEL(p);
  N730_REQUIRE(m->finalized && d_x && d_y, N730_STATE, "run_linear: model not finalized or null buffers");
  N730_REQUIRE(which == 4 || !m->c.stream_depth, N730_STATE, "run_linear: layer weights are host-resident (streamed)");
  const QWeight* w = nullptr;
  if (which == 4) w = m->lm_head;
  else {
    N730_REQUIRE(layer >= 0 && layer < m->c.layers, N730_BAD_ARG, "run_linear: layer %d", layer);
    const Layer& y = m->L[layer];
    w = which == 0 ? y.qkv : which == 1 ? y.o : which == 2 ? y.gate_up : which == 3 ? y.down : nullptr;
  }
  N730_REQUIRE(w, N730_BAD_ARG, "run_linear: which %d", which);
  GemvArgs a = {};
  a.w = w; a.x = d_x; a.ldx = w->cols; a.batch = batch; a.y = d_y;
  a.swiglu = which == 2; a.ldy = which == 2 ? w->rows / 2 : w->rows;
  cudaStream_t st = stream ? (cudaStream_t)stream : m->st;
  if (use_gemm_tc(*w, batch, a.swiglu != 0) && !m->c.exact_gemv) return gemm_tc_launch(a, m->rms_ws, st);  // as the decode step
  return gemv_launch(a, st);
}

// Algorithmic bytes of one linear: packed codes + scale/zero + x + y.
N730_API int64_t n730_model_linear_bytes(void* p, int layer, int which, int batch) {
  Model* m = (Model*)p;
  if (!m || !m->finalized) return -1;
  const QWeight* w = which == 4 ? m->lm_head
                   : (layer < 0 || layer >= m->c.layers) ? nullptr
                   : which == 0 ? m->L[layer].qkv : which == 1 ? m->L[layer].o
                   : which == 2 ? m->L[layer].gate_up : which == 3 ? m->L[layer].down : nullptr;
  if (!w) return -1;
  const int64_t codes = ((int64_t)w->rows * w->cols * w->bits + 7) / 8;
  const int64_t sz = w->bits == 16 ? 0 : (w->sz_mode == 0 ? (int64_t)w->rows * w->n_groups * 4 : 8);  // fp16 s + z
  const int64_t out_rows = which == 2 ? w->rows / 2 : w->rows;
  return codes + sz + (int64_t)batch * (w->cols + out_rows) * 4;
}
