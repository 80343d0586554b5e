/*
 * n730_cuda.h - B200 (sm_100a) kernels and C ABI (library: n730_cuda.so).
 *
 * Part 1 is a drop-in for the reference CUDA library src-code/cpp/n730_cuda.cu
 * (ctypes binding: src-code/inference.py:28-138; also used by
 * src-code/diagnose_binary.py:15-17,257): the same 26 symbols, argument types
 * and return codes (0 OK, -10 CUDA error, -11 out of memory, -12 NULL;
 * n730_cuda.cu:41-44).  Part 2 is the fast path the reference does not have:
 * resident packed weights, the fused dequant-GEMV, paged KV attention and a
 * whole-step decode engine.  New return codes: -13 bad argument, -14
 * unsupported, -15 device wait timed out, -16 wrong state, -17 collective
 * error.  n730_last_error() describes the last failure on the calling thread.
 *
 * Streams: part 1 runs on the legacy default stream and blocks like the
 * reference; part 2 functions take a cudaStream_t as void* (NULL = default).
 */
#ifndef N730_CUDA_H
#define N730_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================= Part 1: reference ABI ======================= */

/* Context with activation / norm / score buffers.  Replaces n730_cuda.cu:362-422. */
int n730_cuda_init(int hidden_size, int num_heads, int head_dim, int vocab_size, int max_seq,
                   int max_weight_elements, void** out_ctx);
/* Replaces n730_cuda.cu:424-442. */
void n730_cuda_destroy(void* ctx);
/* host -> ctx activations [seq, hidden].  Replaces n730_cuda.cu:444-456. */
int n730_load_activations(void* ctx, const float* host_activations, int seq_len, int hidden_size);
/* ctx activations -> host.  Replaces n730_cuda.cu:458-470. */
int n730_get_activations(void* ctx, float* host_out, int seq_len, int hidden_size);
/* Stage one per-tensor packed weight (prec 2/4/8/16) for the next n730_linear*;
 * codes stay packed on the device.  Replaces n730_cuda.cu:472-505. */
int n730_upload_weight(void* ctx, const uint8_t* raw_bytes, int prec_id, int n_elements, float scale,
                       float zero_point);
/* Replaces n730_cuda.cu:507-520. */
int n730_upload_norm_weight(const float* host_w, int n_elements, void** out_ptr);
/* Replaces n730_cuda.cu:522-524. */
void n730_free_device_buf(void* ptr);
/* norm_buf = rmsnorm(activations) * w.  Replaces n730_cuda.cu:526-547. */
int n730_rmsnorm(void* ctx, const float* d_norm_w, int seq_len, float eps);
/* d_out[seq, out] = norm_buf[seq, in] . W^T (fused dequant-GEMV on the staged
 * weight).  Replaces n730_cuda.cu:549-579. */
int n730_linear(void* ctx, float* d_out, int seq_len, int in_dim, int out_dim);
/* Replaces n730_cuda.cu:847-870. */
int n730_linear_from_buf(void* ctx, const float* d_in, float* d_out, int seq_len, int in_dim,
                         int out_dim);
/* activations += delta.  Replaces n730_cuda.cu:581-593. */
int n730_residual_add(void* ctx, const float* d_delta, int seq_len);
/* Replaces n730_cuda.cu:595-608. */
int n730_add_bias(void* ctx, float* d_out, const float* d_bias, int seq_len, int dim);
/* gate = silu(gate) * up.  Replaces n730_cuda.cu:610-622. */
int n730_swiglu(float* d_gate, float* d_up, int seq_len, int intermediate_size);
/* rotate_half RoPE in place.  Replaces n730_cuda.cu:624-640. */
int n730_apply_rope(float* d_x, const float* d_cos, const float* d_sin, int seq_len, int n_heads,
                    int head_dim, int position_offset);
/* fp32 cos/sin tables [max_seq, head_dim/2] (host powf/cosf/sinf).
 * Replaces n730_cuda.cu:642-677. */
int n730_rope_precompute(int max_seq, int head_dim, float theta, void** d_cos_out, void** d_sin_out);
/* Causal mask (seq_q > 1) + softmax rows.  Replaces n730_cuda.cu:679-707. */
int n730_softmax_scores(float* d_scores, int n_heads, int seq_q, int seq_total, int cache_offset);
/* GQA attention over contiguous fp32 K/V [total, n_kv, hd]; probabilities left
 * in the ctx score buffer.  Replaces n730_cuda.cu:709-845. */
int n730_attention_forward(void* ctx, const float* d_q, const float* d_k_cache, const float* d_v_cache,
                           float* d_out, int seq_q, int seq_total, int n_heads, int n_kv_heads,
                           int head_dim, int cache_offset);
/* No counterpart in the reference: n730_attention_forward without a context
 * and without allocating.  The [n_heads, seq_q, seq_total] scores live in a
 * fixed 4 MiB device array (heads * seq_q * seq_total <= 1 Mi floats and
 * seq_q, heads <= 65535, else N730_BAD_ARG); first call per device resolves it (make it outside stream
 * capture); calls that overlap in time race on it.  Runs on `stream`. */
int n730_attention_forward_noalloc(const float* d_q, const float* d_k_cache, const float* d_v_cache,
                                   float* d_out, int seq_q, int seq_total, int n_heads, int n_kv_heads,
                                   int head_dim, int cache_offset, void* stream);
/* Replaces n730_cuda.cu:887-950. */
int n730_attention_qk_only(void* ctx, const float* d_q, const float* d_k_cache, int seq_q,
                           int seq_total, int n_heads, int n_kv_heads, int head_dim);
/* ctx scores -> host [n_heads, seq_q, seq_total].  Replaces n730_cuda.cu:872-885. */
int n730_get_scores(void* ctx, float* h_out, int n_heads, int seq_q, int seq_total);
/* Replaces n730_cuda.cu:953-959. */
int n730_device_alloc(int n_floats, void** out_ptr);
/* Replaces n730_cuda.cu:961-963. */
void n730_device_free(void* ptr);
/* Replaces n730_cuda.cu:965-979. */
int n730_memcpy_d2d(void* dst, const void* src, int n_floats);
int n730_memcpy_h2d(void* dst, const void* src, int n_floats);
int n730_memcpy_d2h(void* dst, const void* src, int n_floats);
/* Replaces n730_cuda.cu:981-984. */
int n730_sync(void);
/* Replaces n730_cuda.cu:986-988. */
const char* n730_cuda_version(void);

/* ======================= Part 2: fast path (new) ======================= */

/* Message for the last non-zero return code on this thread. */
const char* n730_last_error(void);

/* Register a packed weight W[rows, cols] in HBM.  prec_id: 2/4/8/16
 * (per-tensor: scale, zero_point used) or 0x42/0x44/0x48 (group-wise:
 * scales16/zeros16 fp16 [rows, cols/group_size]).  codes use the .n730
 * packing (flattened row-major, element 0 in the low bits).  Sources are host
 * (src_on_device = 0, copied before return) or device pointers.  Rows are
 * re-laid out to 16-byte strides where needed.  Replaces the per-token
 * upload path n730_cuda.cu:472-505 for resident weights. */
int n730_qweight_create(int prec_id, int rows, int cols, int group_size, float scale, float zero_point,
                        const void* codes, const void* scales16, const void* zeros16, int src_on_device,
                        void* stream, void** out_qw);
void n730_qweight_destroy(void* qw);
/* Device layout: 0 row-major (all formats), 1 tensor-core fragment tiles (INT4 group-wise,
 * group % 64 == 0), used by the tensor-core GEMV; dequant and gather read either. */
int n730_qweight_set_layout(void* qw, int layout, void* stream);
/* info[8] = prec, bits, rows, cols, group, n_groups, row_bytes, device bytes. */
int n730_qweight_info(void* qw, int64_t* info);
/* Bit-exact dequant of the whole weight to fp32 d_out[rows, cols]:
 * (float(q) - zero) * scale, the reference formula (n730core.cpp:57-142). */
int n730_dequant_to_f32(void* qw, float* d_out, void* stream);
/* d_out[i, :] = dequantised row d_tokens[i] (embedding gather). */
int n730_embed(void* qw, const int32_t* d_tokens, int n, float* d_out, void* stream);
/* Fused dequant-GEMV: d_y[b, :] = (d_residual[b, :] +) W . xn[b, :] (+ d_bias),
 * xn = rmsnorm(d_x[b, :]) * d_norm_w when d_norm_w != NULL, else d_x.
 * swiglu != 0: rows are interleaved gate/up and d_y[b, r/2] = silu(g) * u.
 * Replaces n730_linear / n730_linear_from_buf + add_bias + residual_add +
 * rmsnorm + swiglu (n730_cuda.cu:526-622,847-870) for resident weights. */
int n730_qlinear(void* qw, const float* d_x, int ldx, int batch, float* d_y, int ldy, const float* d_bias,
                 const float* d_residual, int ldr, const float* d_norm_w, float eps, int swiglu,
                 void* stream);
/* Many-token linear on the tcgen05 tensor cores (TMEM accumulators): the same epilogues as
 * n730_qlinear for `tokens` rows of x; weights must be INT4 in tensor-core fragment tiles
 * (n730_qweight_set_layout 1).  d_ws: `tokens` floats of device workspace when d_norm_w is set.
 * Any token count: 256- / 128-token tiles for prefill, 32 / 64 / 128 for decode batches, K split
 * over CTAs (fixed-order fold) when a decode-sized call would leave SMs idle.  Its internal
 * workspaces grow on the first call of a size (not inside a stream capture).
 * Replaces the per-layer cuBLAS Sgemm of prefill (n730_cuda.cu:549-579, 847-870). */
int n730_qgemm(void* qw, const float* d_x, int ldx, int tokens, float* d_y, int ldy, const float* d_bias,
               const float* d_residual, int ldr, const float* d_norm_w, float eps, int swiglu, float* d_ws,
               void* stream);
/* Next-token sampling on the GPU (replaces the host sampler, inference.py:674-682): for each
 * of `batch` rows of d_logits (row stride ld >= vocab), temperature <= 0 gives the first index
 * of the largest logit; otherwise temperature + nucleus (top_p) sampling with u uniform in
 * [0, 1) from a hash of (seed, counter, row): tokens ordered by probability (ties by index),
 * the nucleus the shortest prefix whose mass reaches top_p, the token the first whose
 * cumulative mass exceeds u times the nucleus mass.  d_tokens [batch] int32 out; d_u [batch]
 * receives u (may be null).  Asynchronous on `stream`. */
int n730_sample(const float* d_logits, int batch, int vocab, int ld, float temperature, float top_p,
                uint64_t seed, uint64_t counter, int32_t* d_tokens, float* d_u, void* stream);
/* Load packed-weight blocks of a .n730 file onto the current device without an intermediate
 * host copy (replaces the per-call Python reads of inference.py:355-366 and the read + dequant
 * of n730core.cpp:192-248): block i at absolute offset offsets[i] becomes out_handles[i] (as
 * n730_qweight_create).  Blocks are read with pread into two page-aligned pinned buffers, so
 * the read of one overlaps the copy and conversion of the previous on `stream`.  Per-tensor
 * ids 2/4/8/16 and group-wise 0x42/0x44/0x48; N730_UNSUPPORTED for a per-tensor block whose
 * payload is not its packed codes.  bytes_read (may be null): block bytes read.  On error no
 * handle is left allocated. */
int n730_qweight_load_blocks(const char* path, int n, const int64_t* offsets, void* stream, void** out_handles,
                             int64_t* bytes_read);
/* Group-wise quantiser on the GPU (the converter's per-group rule):
 * d_w fp32 [rows, cols] -> packed codes, fp16 scales and zeros [rows, cols/group]. */
int n730_quantize_grouped(const float* d_w, int rows, int cols, int bits, int group, uint8_t* d_codes,
                          uint16_t* d_scales16, uint16_t* d_zeros16, void* stream);

/* ---- whole-model engine (replaces N730CudaTransformer.forward's per-op loop,
 * src-code/inference.py:259-669) ---- */
typedef struct N730ModelConfig {
  int32_t hidden, layers, heads, kv_heads, head_dim, ffn, vocab;
  float rms_eps, rope_theta;
  int32_t max_ctx;      /* KV capacity per sequence (positions) */
  int32_t max_batch;    /* sequences decoded together */
  int32_t page_size;    /* KV page size in positions (0 -> 64) */
  int32_t max_prefill;  /* prefill chunk (0 -> 512) */
  int32_t tie_embeddings;
  int32_t tp_rank, tp_size;  /* tensor parallel position (0, 1 for one GPU) */
  int32_t use_graphs;   /* replay the decode step as a CUDA graph */
  int32_t use_pdl;      /* programmatic dependent launch between kernels */
  int32_t exact_gemv;   /* 1: fp32 CUDA-core GEMV everywhere; 0: INT4 g%64 weights use the
                           tensor-core GEMV (x rounded to fp16) */
  int32_t per_op_decode; /* 1: batch-1 decode as one kernel per op; 0: one persistent
                            cooperative kernel for the whole step when the model allows it and its
                            layers average >= 32 MB of weights (smaller layers: the per-op kernels
                            chained with PDL are faster, 0.5B shape 0.86 vs 1.00 ms); -1: the
                            persistent kernel whenever the model allows it */
  int32_t stream_depth;  /* 0: all layer weights resident in HBM.  d > 0: per-layer weights live
                            in pinned host memory and are copied into d + 1 HBM slots on a copy
                            stream, d layers ahead of the layer being computed (the reference's
                            N730Scheduler prefetch, scheduler.py:236-287, as host->HBM copies) */
  int32_t ffn_fuse;      /* persistent decode: 0 runs gate|up and down_proj as ONE phase (each CTA owns
                            whole FFN quant groups, down_proj partial sums reduced in a fixed order)
                            when the down groups divide evenly over the SMs, or when the two-phase
                            FFN does not fit the kernel (72B); 1 whenever the shapes allow it;
                            -1 never (two GEMV phases) */
  int32_t tp_allreduce;  /* tensor parallel, decode-sized row-split sums: 0 one-shot over peer memory
                            (CUDA IPC, after n730_model_tp_ipc_open), fused with the residual add;
                            1 NCCL allreduce always */
  int32_t kv_pool_pages; /* pages in the KV pool shared by the sequences (0: max_batch x pages per
                            sequence); a sequence takes pages as it grows and returns them when
                            released (n730_model_seq_release) */
} N730ModelConfig;

/* weight slots (n730_model_set_qweight); EMBED/LMHEAD take layer = -1 */
enum { N730_W_Q = 0, N730_W_K = 1, N730_W_V = 2, N730_W_O = 3, N730_W_GATE = 4, N730_W_UP = 5,
       N730_W_DOWN = 6, N730_W_EMBED = 7, N730_W_LMHEAD = 8 };
/* vector slots (n730_model_set_vector); FINAL_NORM takes layer = -1; absent norms are ones */
enum { N730_V_INPUT_NORM = 0, N730_V_POST_NORM = 1, N730_V_Q_BIAS = 2, N730_V_K_BIAS = 3, N730_V_V_BIAS = 4,
       N730_V_O_BIAS = 5, N730_V_GATE_BIAS = 6, N730_V_UP_BIAS = 7, N730_V_DOWN_BIAS = 8, N730_V_FINAL_NORM = 9 };

int n730_model_create(const N730ModelConfig* cfg, void** out_model);
void n730_model_destroy(void* model);
/* The model takes ownership of qw (q/k/v and gate/up are fused at finalize). */
int n730_model_set_qweight(void* model, int layer, int slot, void* qw);
int n730_model_set_vector(void* model, int layer, int slot, const float* data, int n, int on_device);
/* Fuse weights, build RoPE tables, the paged KV pool and workspaces. */
int n730_model_finalize(void* model);
/* Clear every sequence's KV (the reference's kv.clear(), inference.py:251-252). */
int n730_model_reset(void* model);
int n730_model_seq_len(void* model, int seq);
/* Take positions [0, len) of sequence seq as already cached (resume / benchmark positioning). */
int n730_model_set_seq_len(void* model, int seq, int len);
/* Append n tokens to sequence seq; logits [vocab] of the last position to host.
 * Same contract as N730CudaTransformer.forward (inference.py:467-669). */
int n730_model_forward(void* model, int seq, const int32_t* host_tokens, int n, float* host_logits);
/* One decode step for sequences [0, batch): host ids in, host logits [batch][vocab] out. */
int n730_model_decode(void* model, const int32_t* host_tokens, int batch, float* host_logits);
/* Page-locked host memory (no counterpart in the reference): a logits buffer from here (or
 * registered with cudaHostRegister) receives n730_model_decode's copy directly, with no
 * staging copy through the engine's own buffer. */
int n730_host_alloc(size_t bytes, void** out);
int n730_host_free(void* ptr);
/* The same step followed by GPU sampling (n730_sample with counter = the number of sampled
 * steps so far): host ids in, host next-token ids [batch] out (4 bytes per sequence cross
 * the bus instead of the logits).  host_u [batch] receives the uniform draws (may be null). */
int n730_model_decode_sample(void* model, const int32_t* host_tokens, int batch, float temperature, float top_p,
                             uint64_t seed, int32_t* host_next, float* host_u);
/* Same step with device-resident ids/logits, asynchronous on `stream`. */
int n730_model_decode_device(void* model, const int32_t* d_tokens, int batch, float* d_logits, void* stream);
/* Self-check of the bounded peer wait of the one-shot allreduce (no counterpart in the
 * reference): one op as rank 0 of 2 with a local stand-in for rank 1's region.  peer_arrives 0:
 * the wait runs out after wait_ns and N730_TIMEOUT (-15) comes back through the device error
 * word, the context stays usable; 1: the peer's slice is present and the op returns 0 with the
 * sum checked. */
int n730_tp_wait_check(int64_t wait_ns, int peer_arrives, void* stream);
/* Release a sequence (its KV pages return to the pool, its length becomes 0). */
int n730_model_seq_release(void* model, int seq);
/* Move sequence src (page ids, length) into the empty slot dst (no KV data moves); src becomes
 * empty.  Decode steps run slots [0, batch): finished sequences are replaced by the last. */
int n730_model_seq_move(void* model, int dst, int src);
/* KV page pool: free and total pages. */
int n730_model_kv_pages(void* model, int* free_pages, int* total_pages);
/* info[16]: weight bytes, KV bytes per position, KV capacity bytes, splits, qkv dim, pages/seq, finalized,
 * persistent batch-1 decode, untied embedding bytes, streamed bytes per pass, FFN fused, phase table in
 * global memory, tensor-parallel plan mismatch (every rank fell back to per-op), persistent grid. */
int n730_model_info(void* model, int64_t* info);
void* n730_model_stream(void* model);
/* One resident linear alone (which: 0 q|k|v, 1 o, 2 gate|up + SwiGLU, 3 down, 4 lm_head),
 * no norm/bias/residual; used to time the dequant-GEMV on the model's weights. */
/* Tensor parallelism (config tp_rank / tp_size > 1; no counterpart in the reference): every
 * rank holds a shard - q/k/v by heads, gate/up by FFN rows in whole quant groups, o/down by
 * the matching input columns, lm_head by vocabulary rows (or replicated) - and the row-split
 * projections' partial sums are allreduced (NCCL) before the residual add.  Rank 0 makes the
 * id, the host shares it, every rank calls tp_init before finalize. */
int n730_tp_unique_id(uint8_t* out_128_bytes);
int n730_model_tp_init(void* model, const uint8_t* id_128_bytes, int rank, int size);
/* One-shot allreduce over NVLink peer memory (config tp_allreduce 0; no counterpart in the
 * reference, which has no multi-GPU path): after tp_init every rank exports its exchange region
 * (N730_IPC_HANDLE_BYTES bytes), the host gathers all ranks' handles in rank order, and every
 * rank opens them (collective; the host barriers before the first step).  Decode-sized
 * row-split sums then bypass NCCL: push to every rank, bounded flag wait, rank-order sum. */
#define N730_IPC_HANDLE_BYTES 64
int n730_model_tp_ipc_handle(void* model, uint8_t* out_handle);
int n730_model_tp_ipc_open(void* model, const uint8_t* handles, int size);
/* Launch only the persistent kernel of a batch-1 decode step (no embedding, no
 * position update; repeated calls recompute the same position).  Timing hook;
 * N730_UNSUPPORTED (-14) when the model decodes with one kernel per op. */
int n730_model_run_step_kernel(void* model, void* stream);
/* The same launch with per-phase timing (profiling hook, no counterpart in the reference):
 * host_times [6 n_phases + 1][grid] per CTA (row 6p: arrival at the barrier before phase p,
 * 6p+1: departure from it, 6p+2/6p+3: marks inside the phase, 6p+4/6p+5: ns its warps waited
 * for weight chunks, last row: end of the last phase; %globaltimer ns), host_kinds
 * [n_phases] (0 GEMV, 1 attention, 2 FFN).  host_times null: only *n_phases and *grid. */
int n730_model_trace_step(void* model, void* stream, uint64_t* host_times, int64_t cap, int8_t* host_kinds,
                          int* n_phases, int* grid);
/* One of the model's linears alone (which: 0 q|k|v, 1 o_proj, 2 gate|up + SwiGLU, 3 down_proj,
 * 4 lm_head) on `batch` device rows, with the kernel the decode step picks for that batch
 * (tensor-core GEMV, or the tcgen05 GEMM from 9 rows for linears whose grid fills the SMs, any from 128). */
int n730_model_run_linear(void* model, int layer, int which, const float* d_x, int batch, float* d_y,
                          void* stream);
/* Algorithmic bytes of that linear for `batch` rows: codes + fp16 scale/zero + x + y. */
int64_t n730_model_linear_bytes(void* model, int layer, int which, int batch);

#ifdef __cplusplus
}
#endif
#endif
