/*
 * vxb.h -- C ABI of vortex_b200, the B200 (sm_100a) implementation of the
 * Vortex quantized-inference hot path.
 *
 * Conventions
 *  - Every entry point returns an int status: VXB_OK (0) or a negative VXB_E*
 *    code; none aborts or throws. vxb_last_error() gives the message, which
 *    maps onto the reference's `Err(String)` results.
 *  - Buffers are caller-owned. Pointers named d_* are device pointers (from
 *    vxb_alloc, cudaMalloc or any allocator of the same device); h_* are host
 *    pointers. `stream` is a cudaStream_t passed as void* (NULL = default).
 *  - One context per device. A context is not shared between host threads
 *    without external locking (the reference serialises its handle tables
 *    with a Mutex; callers keep that discipline).
 *  - bf16 / f16 values are passed as uint16_t bit patterns.
 *
 * Each declaration names the reference interface it replaces
 * (MangoByteLabs/vortex, paths relative to that project).
 */
#ifndef VXB_H
#define VXB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VXB_ABI_VERSION 1

/* status codes */
#define VXB_OK 0
#define VXB_EINVAL (-1)      /* bad argument (shape, pointer, enum) */
#define VXB_ECUDA (-2)       /* CUDA runtime error */
#define VXB_ENOMEM (-3)      /* device or host allocation failed */
#define VXB_ETIMEOUT (-4)    /* a bounded device-side wait ran out */
#define VXB_EFORMAT (-5)     /* malformed GGUF data */
#define VXB_ENOBLOCKS (-6)   /* KV cache out of blocks */
#define VXB_EUNSUPPORTED (-7)/* valid request the library does not handle */
#define VXB_ENCCL (-8)       /* NCCL error */

/* weight block formats: the GGML type ids of gguf_loader.rs GGMLQuantType
 * (src/gguf_loader.rs:61-75) */
#define VXB_Q4_0 2
#define VXB_Q8_0 8
/* further GGUF tensor types (dequantize, upload and GEMV over their raw
 * rows; the tiled kernels take Q4_0 / Q8_0) */
#define VXB_GGML_F32 0
#define VXB_GGML_F16 1
#define VXB_Q4_1 3

/* element types */
#define VXB_F32 0
#define VXB_BF16 1
#define VXB_F16 2
#define VXB_I8 3

typedef struct vxb_ctx vxb_ctx;

/* ------------------------------------------------------------------------ */
/* Context and memory.                                                       */
/* Replaces gpu_runtime::CpuRuntime alloc/free/copy                          */
/* (src/gpu_runtime.rs:297-348) and cuda_available (src/gpu_runtime.rs:654). */
/* ------------------------------------------------------------------------ */
int vxb_abi_version(void);
int vxb_device_count(int *count);
int vxb_init(int device, vxb_ctx **out);
int vxb_destroy(vxb_ctx *ctx);
const char *vxb_last_error(const vxb_ctx *ctx); /* ctx may be NULL: last global error */
int vxb_alloc(vxb_ctx *ctx, size_t bytes, void **d_out);
int vxb_free(vxb_ctx *ctx, void *d_ptr);
int vxb_memcpy_h2d(vxb_ctx *ctx, void *d_dst, const void *h_src, size_t bytes, void *stream);
int vxb_memcpy_d2h(vxb_ctx *ctx, void *h_dst, const void *d_src, size_t bytes, void *stream);
int vxb_memset(vxb_ctx *ctx, void *d_dst, int value, size_t bytes, void *stream);
int vxb_sync(vxb_ctx *ctx, void *stream);
/* Synchronize the device, read and clear the device error words: the
 * context's own and the one in vxb_gemv_q_static's fixed array on the
 * context's device (shared by every context of that device). Kernels bound
 * every wait (clock64 budget); a wait that runs out sets the word and the
 * kernel finishes instead of hanging. Returns VXB_ETIMEOUT (and *out != 0)
 * when that happened since the last call. Allocates nothing. */
int vxb_device_error(vxb_ctx *ctx, int *out);
/* Self-test of the bounded waits above (no counterpart in the reference; the
 * timeout semantics follow the heartbeat timeouts of dist_runtime.rs:426-456):
 * runs the library's own wait helper - kind 0 the mbarrier wait of the stage
 * rings, kind 1 the peer-slot poll of the one-shot all-reduce - on a barrier
 * nobody arrives on / a slot nobody fills, with a budget of budget_cycles SM
 * clocks (1 .. 2^31). The wait gives up, sets the error word (static_word = 0:
 * the context's, 1: the one in vxb_gemv_q_static's fixed array) and the
 * kernel returns, so the next vxb_device_error reports VXB_ETIMEOUT. */
int vxb_selftest_wait_timeout(vxb_ctx *ctx, int kind, int static_word, long long budget_cycles, void *stream);

/* ------------------------------------------------------------------------ */
/* Weight blocks (host codec).                                               */
/* The storage format is the GGUF block layout of gguf_loader.rs             */
/* (Q8_0: f16 d + 32 x i8; Q4_0: f16 d + 16 bytes, byte j = elements 2j (low  */
/* nibble) and 2j+1 (high), value = nibble - 8; src/gguf_loader.rs:413-498). */
/* Codes follow QuantTensor::quantize PerGroup rules with group 32 over the  */
/* flat buffer (src/quantize.rs:96-163, calibration 585-600); the f64 scale  */
/* is narrowed to f32 and then to f16 by tensor_engine::f32_to_f16           */
/* (truncating, src/tensor_engine.rs:42-64).                                 */
/* ------------------------------------------------------------------------ */
size_t vxb_block_bytes(int fmt, size_t n_elements);
/* Replaces QuantTensor::quantize (src/quantize.rs:81-163) + pack_int4 (664). */
int vxb_pack_blocks_f64(int fmt, const double *h_w, size_t n, uint8_t *h_blocks);
int vxb_pack_blocks_f32(int fmt, const float *h_w, size_t n, uint8_t *h_blocks);
/* Replaces dequantize_q4_0 / dequantize_q4_1 / dequantize_q8_0 /
 * dequantize_f16 / copy_f32 (src/gguf_loader.rs:413-531): fmt any of the
 * GGUF types above (vxb_block_bytes gives their sizes). */
int vxb_unpack_blocks(int fmt, const uint8_t *h_blocks, size_t n, float *h_out);

/* Device quantizer: f32 weights on the device -> GGUF blocks on the device,
 * bit-identical to vxb_pack_blocks_f32. Replaces QuantTensor::quantize for
 * weights that already live in HBM. */
int vxb_quantize_blocks(vxb_ctx *ctx, int fmt, const float *d_w, size_t n, uint8_t *d_blocks,
                        void *stream);
/* Device dequantizer (the gguf_loader.rs dequantizers on the device, every
 * GGUF type above; bit-identical with vxb_unpack_blocks). */
int vxb_dequantize_blocks(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, size_t n, float *d_out,
                          void *stream);

/* ------------------------------------------------------------------------ */
/* QuantTensor codes (the quantize / dequantize / quantized_matmul builtins, */
/* src/interpreter.rs:7278-7346): INT8 = one two's-complement byte per      */
/* element, INT4 = two per byte (pack_int4, low nibble = even flat index,   */
/* src/quantize.rs:664-672). Scales are f64, zero points 0 (symmetric).     */
/* ------------------------------------------------------------------------ */
#define VXB_QT_INT8 0
#define VXB_QT_INT4 1
size_t vxb_qt_data_bytes(int fmt, size_t n);
size_t vxb_qt_num_groups(size_t n, size_t group_size); /* group_size 0: PerTensor (1 scale) */
/* QuantTensor::quantize for INT8 / INT4 (src/quantize.rs:81-163): PerGroup
 * over the flat buffer when group_size > 0, else PerTensor; scale =
 * calibrate_minmax / calibrate_minmax_range (585-600); code =
 * clamp(round(v / scale)). h_scales / h_zero_points hold num_groups entries. */
int vxb_qt_quantize(int fmt, const double *h_data, size_t n, size_t group_size, uint8_t *h_packed,
                    double *h_scales, int64_t *h_zero_points);
/* QuantTensor::get_scale (src/quantize.rs:534-545): the mean of the group
 * scales, summed in order (1.0 for none). */
int vxb_qt_mean_scale(const double *h_scales, size_t n_scales, double *out);
/* QuantTensor::matmul for INT8 x INT8 and INT4 x INT4 (matmul_int8 /
 * matmul_int4, src/quantize.rs:447-515) on the device: A [M, K] and B [K, N]
 * code buffers (row-major), out f64 [M, N] = (f64)(i32 wrapping sum of
 * (a - a_zero_point)(b - b_zero_point)) * a_scale * b_scale. Bit-exact with
 * the reference. Other format pairs: VXB_EUNSUPPORTED. */
int vxb_quant_matmul(vxb_ctx *ctx, int fmt, const uint8_t *d_a, const uint8_t *d_b, int M, int K, int N,
                     double a_scale, double b_scale, int64_t a_zero_point, int64_t b_zero_point, double *d_out,
                     void *stream);

/* ------------------------------------------------------------------------ */
/* Tiled weights: the kernels' HBM layout of a weight matrix W [N, K]         */
/* (row-major, K % 32 == 0). The same codes and f16 scales as the GGUF       */
/* blocks, regrouped so that each warp reads 512 contiguous bytes per load    */
/* and each lane's 16 bytes are its tensor-core operand fragments. The        */
/* conversion is lossless: vxb_untile_weights restores the exact blocks.     */
/* ------------------------------------------------------------------------ */
size_t vxb_tiled_bytes(int fmt, int N, int K);
int vxb_tile_weights(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, int N, int K, void *d_tiled,
                     void *stream);
int vxb_untile_weights(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K,
                       uint8_t *d_blocks, void *stream);

/* ------------------------------------------------------------------------ */
/* K1: decode dequant-GEMV / skinny GEMM, y[b, n] = sum_k W[n, k] x[b, k].   */
/* Replaces weight_only_matmul (src/quantize.rs:845-852) and the matmul in   */
/* Linear::forward (src/transformer.rs:332-352) for batch <= 32 rows.        */
/* x: bf16 [batch, K]; y: [batch, N] of y_dtype (VXB_F32 or VXB_BF16).        */
/* Accumulates in f32; uses the context workspace for split-K partials.      */
/* ------------------------------------------------------------------------ */
int vxb_gemv_q(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x,
               int batch, int y_dtype, void *d_y, void *stream);
/* The same product over a tensor kept as its GGUF rows (row n = the blocks
 * of W[n, :], vxb_block_bytes(type, K) bytes), for every GGUF type above
 * (F32, F16, Q4_0, Q4_1, Q8_0; K % 32 == 0 for the block types): the weights
 * are the reference's dequantized f32 values (src/gguf_loader.rs:413-531),
 * accumulated in f32. Any batch >= 1. */
int vxb_gemv_blocks(vxb_ctx *ctx, int type, const void *d_rows, int N, int K, const uint16_t *d_x, int batch,
                    int y_dtype, void *d_y, void *stream);
/* The same GEMV for callers that cannot allocate device memory (no
 * counterpart in the reference: it exists for embedders whose runtime owns
 * all device memory, or that must not add allocations mid-run). Scratch lives
 * in a fixed 8 MiB + 64 KiB array in the library, held on every GPU that
 * loads it; limit: batch * round_up(N, 16) <= 1048576, else VXB_EINVAL. Calls
 * share that array: calls that overlap on the GPU race. The first call on a
 * device resolves the array's address (make it before any stream capture).
 * Allocates nothing: no cudaMalloc / cudaFree. */
int vxb_gemv_q_static(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x,
                      int batch, int y_dtype, void *d_y, void *stream);
/* What a GEMV of this shape launches (no counterpart in the reference; a
 * diagnostic of the planner): *kernel 0 = per-warp stream kernel, 1 = group
 * kernel, 2 = tcgen05 kernel; *splits = k-splits per row group; *cluster = 1
 * when the splits add through distributed shared memory, 0 when they add
 * through global partials (splits > 1) or do not split. is_static selects
 * the plan of vxb_gemv_q_static (its splits are capped by its fixed array). */
int vxb_gemv_plan_info(vxb_ctx *ctx, int fmt, int N, int K, int batch, int is_static, int *kernel, int *splits,
                       int *cluster);

/* ------------------------------------------------------------------------ */
/* Paged KV cache. Replaces PagedKVCache (src/kv_cache.rs:29-93) and the     */
/* kv_cache_* builtins (src/kv_cache.rs:183-290). Blocks of block_size       */
/* tokens come from a free stack initialised to (0..max_blocks).rev();       */
/* each (layer, seq_id) has its own block table; a block is popped when the  */
/* last block is full. A token holds [num_kv_heads, head_dim] keys and       */
/* values, stored as bf16 (VXB_BF16) or int8 with one f32 scale per (token,  */
/* head) (VXB_I8: calibrate_minmax absmax/127, src/quantize.rs:585-591).     */
/* Calls on one cache are stream-ordered by the caller.                      */
/* ------------------------------------------------------------------------ */
typedef struct vxb_kv vxb_kv;
/* PagedKVCache::new (src/kv_cache.rs:41-45) / kv_cache_new (183-193) */
int vxb_kv_create(vxb_ctx *ctx, int num_layers, int num_kv_heads, int head_dim, int block_size,
                  int max_blocks, int max_seqs, int max_blocks_per_seq, int kv_dtype, vxb_kv **out);
int vxb_kv_destroy(vxb_kv *kv);
/* PagedKVCache::append_kv (src/kv_cache.rs:54-67) for one token of each of n
 * sequences; d_k / d_v are bf16 [n, num_kv_heads, head_dim]. */
int vxb_kv_append(vxb_kv *kv, int layer, int n, const int64_t *h_seq_ids, const uint16_t *d_k,
                  const uint16_t *d_v, void *stream);
/* n_tokens consecutive tokens of one sequence (prefill), [n_tokens, H, D]. */
int vxb_kv_append_seq(vxb_kv *kv, int layer, int64_t seq_id, int n_tokens, const uint16_t *d_k,
                      const uint16_t *d_v, void *stream);
/* PagedKVCache::free_seq (src/kv_cache.rs:82-89): all layers of seq_id. A
 * block shared with a forked sequence returns to the free stack when the
 * last sequence holding it is freed. */
int vxb_kv_free_seq(vxb_kv *kv, int64_t seq_id);
/* Prefix reuse (the prefix_cache the reference declares but never fills,
 * src/kv_cache.rs:37, 44): the empty sequence dst_seq starts as the first
 * n_tokens tokens of src_seq in every layer. Full blocks are shared (counted
 * once in kv_stats), a partly filled last block is copied; appends to either
 * sequence never touch a shared block. Synchronous on `stream`. */
int vxb_kv_fork(vxb_kv *kv, int64_t src_seq, int64_t dst_seq, int64_t n_tokens, void *stream);
/* kv_cache_stats (src/kv_cache.rs:220-230): out6 = {used_blocks, free_blocks,
 * block_size, num_seqs (tables), device bytes in use, distinct sequences}. */
int vxb_kv_stats(const vxb_kv *kv, int64_t *out6);
int vxb_kv_seq_len(const vxb_kv *kv, int layer, int64_t seq_id, int64_t *len);
int vxb_kv_block_table(const vxb_kv *kv, int layer, int64_t seq_id, int32_t *h_out, int cap, int *n);
/* PagedKVCache::get_kv (src/kv_cache.rs:69-80): f32 [len, H, D] (dequantized). */
int vxb_kv_gather(vxb_kv *kv, int layer, int64_t seq_id, float *d_k_out, float *d_v_out, void *stream);

/* ------------------------------------------------------------------------ */
/* K4: decode attention. Replaces paged_attention / kv_cache_attention       */
/* (src/kv_cache.rs:95-112, 207-218): for query row i (sequence h_seq_ids[i])*/
/* and q head j, out = softmax(q . K^T * softmax_scale) V over every cached   */
/* token of that sequence (no mask), with kv head j / (Hq / Hkv). An empty    */
/* sequence gives zeros, as the reference. q / out are bf16 [n, Hq, D];      */
/* d_lse (optional) receives the natural-log sum of exponentials [n, Hq].    */
/* ------------------------------------------------------------------------ */
int vxb_decode_attention(vxb_kv *kv, int layer, int n, const int64_t *h_seq_ids, const uint16_t *d_q,
                         int num_q_heads, float softmax_scale, uint16_t *d_out, float *d_lse,
                         void *stream);

/* ------------------------------------------------------------------------ */
/* K2: prefill GEMM. Replaces weight_only_matmul (src/quantize.rs:845-852)  */
/* and Linear::forward (src/transformer.rs:332-352) for many rows:           */
/* y[m, n] = sum_k deq(W)[n, k] * x[m, k] over tiled weights (as vxb_gemv_q),*/
/* x bf16 [M, K], y f32 or bf16 [M, N]. The weights are expanded per call   */
/* into bf16 parts that sum to each weight exactly (2 for Q4_0, 3 for Q8_0) */
/* in a context-owned scratch of 6*N*K bytes (grown on demand) and          */
/* multiplied on tcgen05 tensor cores.                                       */
/* ------------------------------------------------------------------------ */
int vxb_gemm_q(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int M, int y_dtype,
               void *d_y, void *stream);

/* ------------------------------------------------------------------------ */
/* K3: flash-attention forward (prefill). Replaces flash_attention_forward   */
/* and multi_head_flash_attention (src/flash_attention.rs:53-159, 519-564):  */
/* per head O = softmax(scale * Q K^T, causal mask key > query) V and        */
/* lse = log-sum-exp of the scaled scores (natural log), as the reference's  */
/* second output. Tensors are bf16 [B, S, heads, d] (per batch the          */
/* reference's [N, H*d] rows, heads interleaved); K/V have Hkv heads, query */
/* head h reads kv head h / (H / Hkv). d must be 128 (VXB_EUNSUPPORTED      */
/* otherwise). d_lse (optional) is f32 [B, H, S]. Runs on tcgen05 / TMEM.   */
/* ------------------------------------------------------------------------ */
int vxb_flash_fwd(vxb_ctx *ctx, const uint16_t *d_q, const uint16_t *d_k, const uint16_t *d_v, int B, int H,
                  int Hkv, int S, int d, float scale, int causal, uint16_t *d_o, float *d_lse, void *stream);

/* Flash-attention backward. Replaces flash_attention_backward
 * (src/flash_attention.rs:227-317): with D_i = dO_i . O_i and P_ij =
 * exp(scale q_i.k_j - lse_i) (0 for masked keys), dV_j = sum_i P_ij dO_i,
 * dS_ij = P_ij (dO_i.v_j - D_i) scale, dK_j = sum_i dS_ij q_i, dQ_i = sum_j
 * dS_ij k_j. Tensors as vxb_flash_fwd (bf16 [B, S, heads, 128], lse f32
 * [B, H, S] from the forward); d_dq f32 [B, S, H, 128], d_dk / d_dv f32
 * [B, S, Hkv, 128] (summed over the query heads of each kv head). Tensor
 * cores (mma.sync, f32 accumulate), deterministic (no atomics). */
int vxb_flash_bwd(vxb_ctx *ctx, const uint16_t *d_q, const uint16_t *d_k, const uint16_t *d_v, const uint16_t *d_o,
                  const uint16_t *d_dout, const float *d_lse, int B, int H, int Hkv, int S, int d, float scale,
                  int causal, float *d_dq, float *d_dk, float *d_dv, void *stream);

/* ------------------------------------------------------------------------ */
/* K5: single ops of the Llama-style block (stdlib/ai/transformer.vx).       */
/* ------------------------------------------------------------------------ */
/* layer_norm (RMS form with bias), stdlib/ai/transformer.vx:413-439:
 * out = bf16(x * w / sqrt(mean(x^2) + eps) + b), x f32 [rows, n]. */
int vxb_rmsnorm(vxb_ctx *ctx, const float *d_x, const float *d_w, const float *d_b, int rows, int n,
                float eps, uint16_t *d_out, void *stream);
/* feed_forward gate, stdlib/ai/transformer.vx:591-603: act = bf16(silu(g) * u)
 * with gu = [g | u] f32 [rows, 2*ffn]. */
int vxb_swiglu(vxb_ctx *ctx, const float *d_gu, int rows, int ffn, uint16_t *d_act, void *stream);
/* argmax, stdlib/ai/transformer.vx:1163-1177 (first index of the maximum). */
int vxb_argmax(vxb_ctx *ctx, const float *d_logits, int rows, int vocab, int32_t *d_out, void *stream);
/* rope_embed, stdlib/ai/transformer.vx:442-466, on each of `rows` rows of f32
 * d_x [rows, n]: adjacent pairs (x[2i], x[2i+1]) rotated by
 * theta = d_pos[row] / exp(i * ln(10000) / dim) (d_pos int64 [rows]), an odd
 * last element copied. Rotation in f64, rounded once to f32 into d_out
 * [rows, n] (d_out may be d_x). dim <= 0 is VXB_EINVAL; rows or n of 0 is
 * an empty result (VXB_OK, nothing read or written). */
int vxb_rope(vxb_ctx *ctx, const float *d_x, int rows, int n, const int64_t *d_pos, int dim, float *d_out,
             void *stream);
/* the `rope` builtin, src/interpreter.rs:2368-2373: as vxb_rope with the angle
 * of pair i given as d_angles[i] (f64 [n_angles], the same for every row) and
 * 0 for i >= n_angles, as the builtin pads a short frequency list. */
int vxb_rope_angles(vxb_ctx *ctx, const float *d_x, int rows, int n, const double *d_angles, int n_angles,
                    float *d_out, void *stream);
/* residual add, _vec_add stdlib/ai/transformer.vx:353-366: d_out = d_a + d_b,
 * f32 [n] (d_out may be d_a or d_b); n = 0 is an empty result (VXB_OK). */
int vxb_add(vxb_ctx *ctx, const float *d_a, const float *d_b, size_t n, float *d_out, void *stream);

/* sample_top_p, stdlib/ai/transformer.vx:1179-1260 (with the file's series
 * _exp, 36-80), for each of `rows` rows of f32 logits [rows, vocab]:
 * probabilities of logit / temperature in f64, the exchange-sort order by
 * descending probability, the cutoff where the cumulative sum reaches top_p,
 * and the draw u = ((1664525 * h_seeds[r] + 1013904223) mod 2^31) / 2^31 over
 * the renormalised prefix; d_out[r] gets the token. Bit-matched to the
 * reference (ties included). vocab <= 131072. Synchronous on `stream`. */
int vxb_sample_top_p(vxb_ctx *ctx, const float *d_logits, int rows, int vocab, double temperature, double top_p,
                     const int64_t *h_seeds, int32_t *d_out, void *stream);

/* ContinuousBatcher (src/kv_cache.rs:117-154) and the batcher_* builtins
 * (188-290): max_batch_size slots; add takes the lowest free slot and the
 * next sequence id (ids are never reused) and fails with VXB_ENOBLOCKS
 * "batcher full" when every slot is taken; remove frees a slot (a bad slot is
 * ignored, as the reference); num_active counts the taken slots. */
typedef struct vxb_batcher vxb_batcher;
int vxb_batcher_create(int max_batch_size, vxb_batcher **out);
int vxb_batcher_destroy(vxb_batcher *b);
int vxb_batcher_add(vxb_batcher *b, const uint64_t *h_tokens, size_t n_tokens, int *slot_out);
int vxb_batcher_remove(vxb_batcher *b, int slot);
int vxb_batcher_num_active(const vxb_batcher *b, int *out);
/* the BatchSlot fields of a taken slot (any output may be NULL) */
int vxb_batcher_slot(const vxb_batcher *b, int slot, int64_t *seq_id, int64_t *position, int *is_prefill,
                     int *is_done, size_t *n_tokens);
/* after a step: position += n, is_prefill cleared, is_done set when done != 0 */
int vxb_batcher_advance(vxb_batcher *b, int slot, int64_t n, int done);

/* ------------------------------------------------------------------------ */
/* Tensor-parallel communicator. Replaces the nccl_ffi.rs externs            */
/* (src/nccl_ffi.rs:12-72): NCCL (opened at run time) over NVLink/NVSwitch. */
/* Rank 0 makes the 128-byte unique id, the caller shares it with the other */
/* ranks, every rank joins. Collectives run on the given stream.            */
/* ------------------------------------------------------------------------ */
typedef struct vxb_comm vxb_comm;
int vxb_nccl_unique_id(void *h_out128);
int vxb_comm_init(vxb_ctx *ctx, int nranks, int rank, const void *h_unique_id128, vxb_comm **out);
int vxb_comm_destroy(vxb_comm *comm); /* collective: every rank calls it */
/* In-place sum over ranks of count elements of dtype VXB_F32 or VXB_BF16.
 * f32 messages up to 512 KiB take a one-shot all-reduce over NVLink peer
 * memory (CUDA IPC mappings made at init; sum in rank order, identical bits
 * on every rank); larger ones and bf16 go through NCCL. */
int vxb_allreduce_sum(vxb_comm *comm, void *d_buf, size_t count, int dtype, void *stream);

/* ------------------------------------------------------------------------ */
/* Decoder: Llama-style block stack (stdlib/ai/transformer.vx:958-1156) with  */
/* a paged KV cache, one token per sequence per step (greedy next token).    */
/* Stands behind the transformer_* builtins / TransformerModel::forward call */
/* signatures (src/transformer.rs:773-814) for this architecture.            */
/* ------------------------------------------------------------------------ */
typedef struct vxb_decoder_config {
    int vocab_size, dim, n_layers, n_heads, n_kv_heads, ffn_dim;
    int max_batch;    /* sequences per step, <= 32 */
    int max_seq;      /* tokens per sequence (prompt + generated) */
    float norm_eps;   /* 1e-5 when <= 0 */
    int weight_fmt;   /* VXB_Q4_0 or VXB_Q8_0 */
    int kv_dtype;     /* VXB_BF16 (0 selects it) or VXB_I8 */
    int kv_block_size;/* 16 when <= 0 */
} vxb_decoder_config;
typedef struct vxb_decoder vxb_decoder;
int vxb_decoder_create(vxb_ctx *ctx, const vxb_decoder_config *cfg, vxb_decoder **out);
/* Tensor-parallel decoder over comm's ranks (one process per GPU, every rank
 * calls the same functions with the same arguments): QKV and gate/up are
 * split by output rows (heads), O and down by input columns, followed by an
 * all-reduce (sum) of the residual stream; the LM head is split by vocabulary
 * rows with a distributed argmax. nranks must divide n_heads, n_kv_heads and
 * vocab_size, and dim / nranks, ffn_dim / nranks must be multiples of 32.
 * init_random and set_weight take the full model on every rank and keep the
 * rank's part, so any rank count gives the same model. */
int vxb_decoder_create_tp(vxb_ctx *ctx, const vxb_decoder_config *cfg, vxb_comm *comm, vxb_decoder **out);
int vxb_decoder_destroy(vxb_decoder *d);
/* init_random_weights (stdlib/ai/transformer.vx:661-725): linears and
 * embedding ~N(0, sigma) from a counter-based generator, norms w=1, b=0. */
int vxb_decoder_init_random(vxb_decoder *d, uint64_t seed, float sigma);
/* Load one weight from host memory: layer >= 0: which 0..6 = wq, wk, wv, wo,
 * w1, w2, w3 as GGUF blocks [out, in]; 7..10 = attention-norm w, b, ffn-norm
 * w, b (f32). layer == -1: 0 embedding (bf16 [vocab, dim]), 1/2 final norm
 * w/b (f32), 3 output projection (blocks [vocab, dim]). */
int vxb_decoder_set_weight(vxb_decoder *d, int layer, int which, const void *h_data, size_t bytes);
/* One step through host buffers (synchronous): token h_tokens[i] of sequence
 * h_seq_ids[i] is appended; h_next gets the greedy next token, h_logits
 * (optional) the logits [batch, vocab]. */
int vxb_decoder_step(vxb_decoder *d, int batch, const int64_t *h_seq_ids, const int32_t *h_tokens,
                     int32_t *h_next, float *h_logits);
/* Prompt of n tokens for a new (empty) sequence in one pass: K2 GEMMs over
 * the n rows and the causal K3 flash attention (head_dim 128), K/V of every
 * position cached. h_next / h_logits (optional) get the greedy next token and
 * the last position's logits [vocab]. Synchronous; the same call on every
 * rank with tensor parallelism. */
int vxb_decoder_prefill(vxb_decoder *d, int64_t seq_id, const int32_t *h_tokens, int n, int32_t *h_next,
                        float *h_logits);
/* The same with device token buffers, ordered on `stream`. */
int vxb_decoder_step_device(vxb_decoder *d, int batch, const int64_t *h_seq_ids,
                            const int32_t *d_tokens, int32_t *d_next, void *stream);
int vxb_decoder_logits(vxb_decoder *d, int batch, float *d_out, void *stream);
int vxb_decoder_free_seq(vxb_decoder *d, int64_t seq_id);
/* A new sequence dst_seq continuing from the first n_tokens tokens of src_seq
 * (vxb_kv_fork on the decoder's cache: shared prompt prefixes are stored and
 * attended once per block). The same call on every rank with tensor
 * parallelism. */
int vxb_decoder_fork(vxb_decoder *d, int64_t src_seq, int64_t dst_seq, int64_t n_tokens);
int vxb_decoder_kv(vxb_decoder *d, vxb_kv **out);
int vxb_decoder_stream(vxb_decoder *d, void **out);

/* ------------------------------------------------------------------------ */
/* GGUF reader. Replaces parse_gguf / get_tensor (src/gguf_loader.rs:       */
/* 341-408, 536-584) for the quantized path: the file is memory-mapped (or  */
/* a caller buffer is parsed in place; it must outlive the handle), parse    */
/* errors carry the reference's messages (vxb_last_error(NULL)), and Q4_0 /  */
/* Q8_0 tensors upload as their blocks into the tiled device layout (no f32  */
/* dequantization): rows = product of the dimensions after the first, K =   */
/* the first (fastest) dimension.                                            */
/* ------------------------------------------------------------------------ */
typedef struct vxb_gguf vxb_gguf;
int vxb_gguf_open(const char *path, vxb_gguf **out);
int vxb_gguf_open_memory(const void *data, size_t nbytes, vxb_gguf **out);
int vxb_gguf_close(vxb_gguf *g);
int vxb_gguf_info(const vxb_gguf *g, uint32_t *version, int64_t *n_tensors, int64_t *n_metadata,
                  uint64_t *data_offset, uint64_t *alignment);
/* dims4: the dimensions as stored, padded with 1; h_data: the tensor's bytes
 * inside the mapping (bounds-checked as get_tensor). Any output may be NULL. */
int vxb_gguf_tensor(const vxb_gguf *g, int64_t index, char *name, size_t name_cap, int *ggml_type, int *n_dims,
                    uint64_t *dims4, uint64_t *offset, uint64_t *nbytes, const void **h_data);
int vxb_gguf_find_tensor(const vxb_gguf *g, const char *name, int64_t *index);
int vxb_gguf_meta_int(const vxb_gguf *g, const char *key, int64_t *value);
int vxb_gguf_meta_float(const vxb_gguf *g, const char *key, double *value);
int vxb_gguf_meta_string(const vxb_gguf *g, const char *key, char *out, size_t cap, size_t *len);
int vxb_gguf_upload_tiled(vxb_ctx *ctx, const vxb_gguf *g, int64_t index, void *d_tiled, size_t tiled_bytes,
                          void *stream);
/* Any tensor's bytes as stored in the file (F32, F16, Q4_0, Q4_1, Q8_0 rows
 * of blocks, no conversion) into a device buffer of at least its size;
 * synchronous. For vxb_gemv_blocks and vxb_dequantize_blocks. */
int vxb_gguf_upload(vxb_ctx *ctx, const vxb_gguf *g, int64_t index, void *d_dst, size_t dst_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* f32 GPT-style model of src/transformer.rs:15-841 (TransformerModel):      */
/* embedding + sinusoidal positions, pre-norm layers (LayerNorm 1e-5,        */
/* biased multi-head attention with an optional [S, S] mask, entries < 0.5  */
/* masked to -1e9; GELU feed-forward), final LayerNorm, output projection.  */
/* create = TransformerModel::new (Xavier from the xorshift seed 42);      */
/* parameters in params_vec order; forward = TransformerModel::forward.    */
/* ------------------------------------------------------------------------ */
typedef struct vxb_tmodel_config {
    int vocab_size, d_model, n_heads, n_layers, d_ff, max_seq_len;
} vxb_tmodel_config;
typedef struct vxb_tmodel vxb_tmodel;
int vxb_tmodel_create(vxb_ctx *ctx, const vxb_tmodel_config *cfg, vxb_tmodel **out);
int vxb_tmodel_destroy(vxb_tmodel *m);
int vxb_tmodel_param_count(const vxb_tmodel *m, size_t *n);
int vxb_tmodel_set_params(vxb_tmodel *m, const float *h_params, size_t n);
int vxb_tmodel_get_params(vxb_tmodel *m, float *h_params, size_t n);
/* logits [S, vocab] f32 of S tokens; h_mask [S, S] f32 or NULL. Synchronous. */
int vxb_tmodel_forward(vxb_tmodel *m, const int32_t *h_tokens, int S, const float *h_mask, float *h_logits);

#ifdef __cplusplus
}
#endif
#endif /* VXB_H */
