/*
 * s8b — B200 (sm_100a) kernels for superl8-serve's pipeline-parallel W8A8 decode step.
 *
 * Plain C ABI: device pointers, sizes and a CUDA stream (passed as void*, a cudaStream_t).
 * The caller owns every buffer; apart from the set-up-time s8b_ipc_alloc, no entry point
 * allocates device memory. Entry points that
 * need scratch take a caller-provided workspace and report its size through a *_workspace_size
 * query. Every entry point is stream-ordered, performs no host synchronisation and returns
 * 0 on success or a negative S8B_ERR_* code (s8b_strerror gives the text). A kernel launch
 * failure returns S8B_ERR_CUDA and records the cudaError_t for s8b_last_cuda_error().
 *
 * Citations name the superl8-serve (reference) interface each entry point replaces; the
 * reference binds its kernels through the `superl8` Python package at those call sites.
 *
 * Numerics: every entry point reproduces the CPU oracle (oracle/ in this repository) bit for
 * bit: binary32 operations in a fixed order without FMA contraction, int32 accumulation for
 * integer products, float64 accumulation for the RMSNorm sums of squares.
 */
#ifndef S8B_H_
#define S8B_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------- */
#define S8B_OK 0
#define S8B_ERR_SHAPE (-1)     /* unsupported or inconsistent sizes                        */
#define S8B_ERR_DTYPE (-2)     /* unsupported activation dtype or codec scheme             */
#define S8B_ERR_ALIGN (-3)     /* pointer or leading dimension not aligned as required     */
#define S8B_ERR_CUDA (-4)      /* a CUDA runtime call or kernel launch failed              */
#define S8B_ERR_PEER (-5)      /* peer memory not registered / peer access unavailable     */
#define S8B_ERR_TIMEOUT (-6)   /* a bounded device-side wait gave up (see s8b_flag_status) */
#define S8B_ERR_WORKSPACE (-7) /* workspace missing or smaller than *_workspace_size       */
#define S8B_ERR_ARG (-8)       /* null pointer or invalid argument                         */
#define S8B_ERR_SCRATCH_LIMIT (-9) /* problem needs more than the no-allocation scratch limit */

/* ---- activation dtypes -------------------------------------------------------------- */
#define S8B_BF16 0
#define S8B_FP16 1

/* ---- wire codec schemes (reference names: "fp16", "int8", "int8-had", "int4", "int4-had",
 * "nf4")
 * fp16     : the activation itself, bit-exact (2 bytes/element, no scales)
 * int8     : int8 codes, one fp32 scale per row
 * int8-had : block-128 Hadamard, then int8 with one fp32 scale per row
 * int4     : two's-complement nibbles (low nibble = even element), fp32 scale per 128-group
 * int4-had : block-128 Hadamard, then int4 as above
 * nf4      : 4-bit NormalFloat codes (index into the 16-entry NF4 codebook, nearest entry to
 *            x / absmax, lowest index on ties), nibbles packed as int4, fp32 absmax scale per
 *            128-group                                                                    */
#define S8B_CODEC_FP16 0
#define S8B_CODEC_INT8 1
#define S8B_CODEC_INT8_HAD 2
#define S8B_CODEC_INT4 3
#define S8B_CODEC_INT4_HAD 4
#define S8B_CODEC_NF4 5

const char *s8b_strerror(int code);
int s8b_version(void);
int s8b_last_cuda_error(void);
/* Number of kernels this library has launched in this process (all devices). */
unsigned long long s8b_launch_count(void);

/* Per-token int8 quantization of activations x[M,K]: scale = absmax/127,
 * code = rint(x * (127/absmax)) clamped to +-127; an all-zero row gets scale 1.
 * Replaces the activation-quant half of superl8.linear
 * (superl8serve/layers/linear.py:122).                                                    */
int s8b_quant_rows(const void *x, int dtype, int8_t *q, float *s, int M, int K, void *stream);

/* Fused residual add + RMSNorm + per-token int8 quantization.
 *   x = (residual_in ? h + residual_in : h) rounded to dtype; residual_out = x (nullable);
 *   y = RMSNorm(x) * w (binary32, eps); optional y_out; (q, s) = quant_rows(y).
 * Replaces superl8.rmsnorm (superl8serve/layers/norm.py:51) fused with the activation quant
 * of the following superl8.linear.                                                        */
int s8b_rmsnorm_quant(const void *h, const void *residual_in, void *residual_out,
                      const void *w, float eps, int8_t *q, float *s, void *y_out, int M, int H,
                      int dtype, void *stream);
/* The same with h given as the split-K partials of a tensor-core GEMM (part int32 [C][M][H],
 * out_kind 2, with that GEMM's activation scales xs [M] and weight scales ws [H]):
 * h = dtype((f32(sum_c part[c]) * xs[m]) * ws[n]), exactly the GEMM's bf16 output. part
 * and ws 16-byte aligned, 1 <= C <= 8. No counterpart in the reference. */
int s8b_rmsnorm_quant_split(const int32_t *part, int C, const float *xs, const float *ws,
                            const void *residual_in, void *residual_out, const void *w,
                            float eps, int8_t *q, float *s, void *y_out, int M, int H, int dtype,
                            void *stream);

/* W8A8 GEMM on CUDA cores (dp4a), for small token counts:
 *   acc[m,n] = sum_k xq[m,k]*w[n,k] (int32);  y[m,n] = dtype((float(acc)*xs[m])*ws[n]).
 * out_kind 0: y is dtype [M,N];  out_kind 1: y is int32 [M,N] raw accumulators.
 * K % 16 == 0; xq, w 16-byte aligned. Replaces superl8.linear / gemm_w8a8
 * (superl8serve/layers/linear.py:122; superl8serve/layers/linear.py:9).                  */
int s8b_gemm_w8a8(const int8_t *xq, const float *xs, const int8_t *w, const float *ws, void *y,
                  int out_kind, int M, int N, int K, int dtype, void *stream);

/* W8A8 GEMM on the tensor cores (tcgen05.mma kind::i8, TMA-fed, TMEM accumulators), same
 * arithmetic and outputs as s8b_gemm_w8a8 (out_kind 0 and 1; out_kind 2: split-K partials,
 * see s8b_gemm_tc_split_count), for token counts where the contraction is dense
 * (M >= 16; M > 256 runs in 256-token passes). K % 128 == 0. Split-K partial sums are
 * reduced inside thread-block clusters (distributed shared memory), so the workspace
 * (s8b_gemm_tc_workspace_size bytes, 256-byte aligned, zero-filled once by the caller) only
 * holds a status word: workspace[0] (int32) receives S8B_ERR_TIMEOUT if a bounded wait
 * inside the kernel gave up, after which the caller must re-zero it. The launch carries a
 * programmatic dependency on the preceding kernel in the stream (weights prefetch early;
 * activations, scales and outputs are touched only after that kernel has completed).
 * Replaces superl8.linear / gemm_w8a8 (superl8serve/layers/linear.py:122).               */
size_t s8b_gemm_tc_workspace_size(int M, int N);
/* out_kind 2 of the tensor-core GEMM: no dequantization and no reduction of the split-K
 * partial sums; y is int32 [C][M][N] with C = s8b_gemm_tc_split_count(M, N, K), and
 * sum_c y[c][m][n] is the int32 accumulator. The row kernels below with a _split suffix read
 * that layout directly (they sum, dequantize y = dtype((f32(acc) * xs[m]) * ws[n]) and go
 * on), so the reduction costs no extra launch. No counterpart in the reference. */
int s8b_gemm_tc_split_count(int M, int N, int K);
int s8b_gemm_w8a8_tc(const int8_t *xq, const float *xs, const int8_t *w, const float *ws,
                     void *y, int out_kind, int M, int N, int K, int dtype, void *workspace,
                     size_t workspace_bytes, void *stream);

/* Weight pre-packing for the tensor-core GEMM: W [N, K] row-major int8 -> units of 128 rows x
 * 128 bytes, tile-major, each unit stored as the 128B-swizzled shared-memory image the MMA
 * reads (rows beyond N zero). s8b_gemm_w8a8_tc_packed then streams every CTA's share of the
 * matrix as one contiguous HBM range with plain bulk copies. Packing runs once at load.     */
size_t s8b_tc_packed_bytes(int N, int K);
int s8b_pack_weights_tc(const int8_t *w, int N, int K, int8_t *packed, void *stream);
int s8b_gemm_w8a8_tc_packed(const int8_t *xq, const float *xs, const int8_t *wpacked,
                            const float *ws, void *y, int out_kind, int M, int N, int K,
                            int dtype, void *workspace, size_t workspace_bytes, void *stream);

/* SwiGLU on a merged [gate | up] row (gu is [M, 2F]) followed by per-token int8 quant:
 *   a = dtype(g / (1 + exp(-g))), y = dtype(a * u), (q, s) = quant_rows(y); y_out nullable.
 * Replaces superl8.act_and_mul(x, "silu") (superl8serve/layers/activation.py:24) fused with
 * the activation quant of the down projection.                                            */
int s8b_silu_mul_quant(const void *gu, int M, int F, void *y_out, int8_t *q, float *s,
                       int dtype, void *stream);
/* The same with gu given as GEMM split-K partials (int32 [C][M][2F], xs [M], ws [2F]; see
 * s8b_rmsnorm_quant_split). No counterpart in the reference. */
int s8b_silu_mul_quant_split(const int32_t *part, int C, const float *xs, const float *ws,
                             int M, int F, void *y_out, int8_t *q, float *s, int dtype,
                             void *stream);

/* Decode-branch head processing for a merged qkv row [M, (Hq+2*Hkv)*D]:
 * per-head RMSNorm of q and k (q_norm_w, k_norm_w [D]), RoPE at positions[m] with binary32
 * tables cos/sin [max_pos, D]; K rotated by the orthonormal Hadamard-128, rounded to dtype
 * and written with V as int8 + fp32 scale into the paged stores at
 * slot = block_table[m][pos/bs]*bs + pos%bs (or slot_mapping[m] when non-null);
 * q is rotated by the same Hadamard and quantized per (token, head) into q_i8 [M,Hq,D],
 * q_s [M,Hq]. q_out (nullable) receives the post-RoPE q in dtype.
 * Replaces GQAAttention.forward's q/k norm + superl8.rope + quantize_kv_write_paged
 * (superl8serve/layers/gqa_attention.py:66-74; superl8serve/engine/kv_cache.py:1095-1116).
 * D must be 128.                                                                          */
int s8b_qkv_post(const void *qkv, const int32_t *positions, const float *cos_tab,
                 const float *sin_tab, int max_pos, const void *q_norm_w, const void *k_norm_w,
                 float eps, int M, int Hq, int Hkv, int D, int8_t *q_i8, float *q_s,
                 void *q_out, int8_t *kc, float *ks, int8_t *vc, float *vs,
                 const int32_t *slot_mapping, const int32_t *block_table, int max_blocks,
                 int block_size, int dtype, void *stream);
/* Stage prologue: s8b_rmsnorm_quant on the previous stage's codec payload [T, 2H]
 * (scheme S8B_CODEC_*): the hidden and residual halves are decoded on load exactly as
 * s8b_codec_decode does (inverse Hadamard across a warp for the -had schemes), added, normed
 * and quantized; residual_out [T, H] receives the sum. H % 128 == 0. Identical to
 * s8b_codec_decode + s8b_rmsnorm_quant. Fuses decompress_activation and the unpack of the
 * reference (superl8serve/dist/__init__.py:300, superl8serve/dist/pipeline.py:301-305)
 * with the next layer's input RMSNorm.                                                    */
int s8b_rmsnorm_quant_codec(const void *payload, const float *scales, int scheme,
                            void *residual_out, const void *w, float eps, int8_t *q, float *s,
                            int M, int H, int dtype, void *stream);
/* The same with qkv given as GEMM split-K partials (int32 [C][M][(Hq+2*Hkv)*D], xs [M],
 * ws [(Hq+2*Hkv)*D]; see s8b_rmsnorm_quant_split). No counterpart in the reference. */
int s8b_qkv_post_split(const int32_t *part, int C, const float *xs, const float *ws,
                       const int32_t *positions, const float *cos_tab, const float *sin_tab,
                       int max_pos, const void *q_norm_w, const void *k_norm_w, float eps, int M,
                       int Hq, int Hkv, int D, int8_t *q_i8, float *q_s, void *q_out,
                       int8_t *kc, float *ks, int8_t *vc, float *vs,
                       const int32_t *slot_mapping, const int32_t *block_table, int max_blocks,
                       int block_size, int dtype, void *stream);

/* Quantize-on-write of new K/V rows k, v [T, Hkv, D] into one layer's paged stores
 * kc/vc [num_blocks, Hkv, bs, D] int8, ks/vs [num_blocks, Hkv, bs] fp32 at
 * row (slot/bs*Hkv + h)*bs + slot%bs. rotate_k != 0 applies the Hadamard-128 to K first.
 * Replaces superl8.quantize_kv_write_paged (superl8serve/engine/kv_cache.py:1108-1116). */
int s8b_kv_write_paged(const void *k, const void *v, int8_t *kc, float *ks, int8_t *vc,
                       float *vs, const int32_t *slot_mapping, int T, int Hkv, int D,
                       int block_size, int rotate_k, int dtype, void *stream);

/* Paged int8 GQA decode attention over block tables, for pre-quantized queries
 * (q_i8 [B,Hq,D], q_s [B,Hq] from s8b_qkv_post). out [B, Hq*D] in dtype; out_q/out_s
 * (nullable, together) additionally receive the per-token int8 quantization of the output
 * row (the o_proj input). context_lens[b] >= 1 tokens of row b are attended; max_ctx is an
 * upper bound on every context_lens[b] (sizes the partition grid). Workspace: see
 * s8b_paged_decode_workspace_size; zero-fill it once before first use (its first word is the
 * status word below; the rest needs no initial value, and one workspace serves calls of any
 * shape it is large enough for); launches sharing a workspace must be stream-ordered.
 * D must be 128; block_size a power of two dividing 256.
 * Replaces superl8.attn_paged_decode_cached (superl8serve/engine/kv_cache.py:1190-1201). */
size_t s8b_paged_decode_workspace_size(int B, int Hq, int D, int max_ctx);
/* Byte offset, inside the decode workspace, of an int32 status word: 0, or S8B_ERR_TIMEOUT
 * when a bounded wait on a tensor-core completion barrier gave up (that launch's output is
 * then invalid). It is the workspace's first word for every B and Hq (the function returns
 * 0). Zero-filled with the workspace; it stays set until the caller clears it after reading
 * an error. No counterpart in the reference (its kernels have no bounded waits). */
size_t s8b_paged_decode_status_offset(int B, int Hq);
/* Selects the kernel behind every paged-decode entry point: 0 (default) = the persistent
 * warp-specialized tensor-core kernel (TMA ring, tcgen05 kind::i8 for q.k and p.v) where the
 * shape allows it (block_size >= 8, 16-byte aligned scale arrays), else the per-partition
 * tensor-core kernel; 1 = CUDA-core (dp2a) partition kernel; 2 = per-partition tensor-core
 * kernel. All give bit-identical results. Returns S8B_ERR_ARG for other values. No
 * counterpart in the reference. */
int s8b_set_attention_impl(int impl);
int s8b_paged_decode_q8(const int8_t *q_i8, const float *q_s, const int8_t *kc, const float *ks,
                        const int8_t *vc, const float *vs, const int32_t *block_table,
                        const int32_t *context_lens, void *out, int8_t *out_q, float *out_s,
                        int B, int Hq, int Hkv, int D, int block_size, int max_blocks,
                        int max_ctx, float scale, void *workspace, size_t workspace_bytes,
                        int dtype, void *stream);
/* s8b_paged_decode_q8 for a decode step: the kernel just before this call on `stream` writes
 * the queries and each row's K/V at position context_lens[b] - 1 only, and the block tables,
 * context lengths and older K/V are final before it starts (the write_decode + decode_attn
 * pair of one decode step, superl8serve/layers/gqa_attention.py:180-190). The persistent
 * kernel then starts streaming the partitions before that position while the previous
 * kernel still runs. Results are identical to s8b_paged_decode_q8. Not for prefill rows
 * (their chunk writes many positions). No counterpart in the reference.                  */
int s8b_paged_decode_q8_step(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                             const float *ks, const int8_t *vc, const float *vs,
                             const int32_t *block_table, const int32_t *context_lens, void *out,
                             int8_t *out_q, float *out_s, int B, int Hq, int Hkv, int D,
                             int block_size, int max_blocks, int max_ctx, float scale,
                             void *workspace, size_t workspace_bytes, int dtype, void *stream);
/* Varlen prefill attention over the int8 paged cache (replaces the superl8
 * attn_int8_varlen call of the reference's prefill, superl8serve/dist/pipeline.py:908-984):
 * rows, queries, cache and output exactly as s8b_paged_decode_q8 (row b attends over the
 * first context_lens[b] positions of block-table row b), output identical to it. The rows
 * are grouped into n_row_blocks row blocks, row_blocks[2i] = first row, row_blocks[2i + 1]
 * = row count (1 .. s8b_paged_prefill_block_rows(Hq, Hkv); larger counts are cut there):
 * consecutive rows of one sequence, whose block-table rows are equal; every row in exactly
 * one block. Each block's K/V partitions are read once for all its rows (a row's heads are
 * columns of the tensor-core tiles). Workspace as s8b_paged_decode_q8.                   */
int s8b_paged_prefill_block_rows(int Hq, int Hkv);
int s8b_paged_prefill_q8(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                         const float *ks, const int8_t *vc, const float *vs,
                         const int32_t *block_table, const int32_t *context_lens,
                         const int32_t *row_blocks, int n_row_blocks, void *out, int8_t *out_q,
                         float *out_s, int B, int Hq, int Hkv, int D, int block_size,
                         int max_blocks, int max_ctx, float scale, void *workspace,
                         size_t workspace_bytes, int dtype, void *stream);

/* No-allocation form of s8b_paged_decode_q8, for callers that cannot allocate device
 * memory: a host-language binding (cgo, JNI, ctypes) that is handed device buffers but owns no
 * allocator, or a serving runtime that reserved all of HBM up front (KV pool sized to fill
 * the GPU) and must not call cudaMalloc on the decode path, where it could fail or stall the
 * device. It takes no workspace: the partition partials live in a fixed 16 MiB array in the
 * library's device memory (held on every GPU that loads the library, until exit). Requests
 * needing more than that, i.e. B*Hq*ceil(max_ctx/256)*(D+2)*4 bytes > 16 MiB, return
 * S8B_ERR_SCRATCH_LIMIT without launching. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture. All calls share the one array, so calls that overlap on the GPU
 * (different streams, or different host threads on the same device) race; serialize them.
 * The array keeps the last call's contents. Its layout is a workspace's: the status word
 * first (see s8b_paged_decode_noalloc_status), then the completion counters of the
 * per-partition kernels, which every call zeroes before it launches them (a stream-ordered
 * memset), then the partials, which are written before they are read. So a call never
 * depends on what an earlier call of another shape, or one that gave up, left behind.
 * It calls no cudaMalloc / cudaFree or other allocating routine.
 * This entry point has no counterpart in the reference.                                   */
int s8b_paged_decode_q8_noalloc(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                                const float *ks, const int8_t *vc, const float *vs,
                                const int32_t *block_table, const int32_t *context_lens,
                                void *out, int8_t *out_q, float *out_s, int B, int Hq, int Hkv,
                                int D, int block_size, int max_blocks, int max_ctx, float scale,
                                int dtype, void *stream);
/* Status word of the no-allocation entry point on the current device: stores the word's value
 * in *previous and replaces it with `replace_with` (0 clears it). The word is 0, or
 * S8B_ERR_TIMEOUT once a bounded wait of a call gave up (that call's output is invalid); it
 * stays set until replaced. Call it after synchronizing the streams the decode calls ran on:
 * it reads and writes with plain synchronous copies. It allocates nothing.
 * No counterpart in the reference (its kernels have no bounded waits).                    */
int s8b_paged_decode_noalloc_status(int32_t *previous, int32_t replace_with);

/* Same attention with the reference's query layout: q [B, Hq, D] in dtype (rotated and
 * quantized internally into the workspace, which must be zero-filled once likewise).
 * out [B, Hq, D] in dtype.                                                                */
size_t s8b_paged_decode_ref_workspace_size(int B, int Hq, int D, int max_ctx);
int s8b_paged_decode(const void *q, const int8_t *kc, const float *ks, const int8_t *vc,
                     const float *vs, const int32_t *block_table, const int32_t *context_lens,
                     void *out, int B, int Hq, int Hkv, int D, int block_size, int max_blocks,
                     int max_ctx, float scale, void *workspace, size_t workspace_bytes,
                     int dtype, void *stream);

/* Token embedding gather: out[m] = table[ids[m]] ([V, H] in dtype).
 * Replaces VocabEmbedding.forward (superl8serve/layers/embedding.py:60-69).               */
int s8b_embed(const int32_t *ids, const void *table, int M, int H, void *out, int dtype,
              void *stream);

/* Greedy sampling: out[m] = argmax_v logits[m, v] (lowest index on ties).
 * Replaces the all-greedy Sampler fast path (superl8serve/layers/sampler.py:51-63).       */
int s8b_argmax(const void *logits, int M, int V, int32_t *out, int dtype, void *stream);

/* The library's binary32 exponential (softmax weights, partition merge, SiLU), elementwise:
 * y[i] = exp_s8b(x[i]). A numerics check of the CPU definition, not a reference seam.      */
int s8b_exp_f32(const float *x, float *y, long long n, void *stream);

/* Inter-stage codec. Rows are the concatenation [a | b] of a [T, Da] and b [T, Db]
 * (b nullable, Db = 0), i.e. the pipeline's packed (hidden, residual) boundary
 * (superl8serve/dist/pipeline.py:246-250). (Da+Db) % 128 == 0 for the int4 / -had schemes.
 * payload: fp16 -> dtype [T, D]; int8* -> int8 [T, D]; int4* -> uint8 [T, D/2].
 * scales : int8* -> fp32 [T]; int4* -> fp32 [T, D/128]; fp16 -> unused.
 * payload / scales may be peer pointers (another GPU's memory, peer access enabled or IPC
 * mapped): the encoder then stores straight across NVLink.
 * Replace superl8.compress_activation / decompress_activation as bound in send / recv
 * (superl8serve/dist/__init__.py:189,300).                                                */
size_t s8b_codec_payload_bytes(int T, int D, int scheme, int dtype);
size_t s8b_codec_scale_count(int T, int D, int scheme);
int s8b_codec_encode(const void *a, const void *b, int T, int Da, int Db, int scheme,
                     void *payload, float *scales, int dtype, void *stream);
int s8b_codec_decode(const void *payload, const float *scales, int T, int Da, int Db,
                     int scheme, void *out_a, void *out_b, int dtype, void *stream);
/* Stage epilogue: s8b_codec_encode with the `a` half given as a GEMM's split-K partials
 * (int32 [C][T][Da], token scales xs [T], row scales ws [Da]; summed and dequantized on load
 * exactly as the GEMM's own output would be), so a stage's last down projection goes
 * straight into the boundary codes. Da % 4 == 0, C <= 8. Codes are identical to the unfused
 * GEMM + s8b_codec_encode. Fuses the boundary pack and compress_activation of the reference
 * (superl8serve/dist/pipeline.py:246-250, superl8serve/dist/__init__.py:189).              */
int s8b_codec_encode_split(const int32_t *part, int C, const float *xs, const float *ws,
                           const void *b, int T, int Da, int Db, int scheme, void *payload,
                           float *scales, int dtype, void *stream);

/* ---- stage-to-stage signalling (no counterpart call in the reference, whose send()
 * synchronises the host instead: superl8serve/dist/__init__.py:243-247) ---------------------
 * A flag is a uint32 in device memory, usually the consumer's, written by the producer across
 * NVLink. Values are epochs read from device memory (*value + add), so a captured CUDA graph
 * replays with fresh values. s8b_flag_set stores the epoch with release semantics at system
 * scope after all prior work on the stream. s8b_flag_wait spins, stream-ordered on the
 * device, until (int32)(*flag - epoch) >= 0 or about timeout_ns nanoseconds pass; on timeout
 * it writes S8B_ERR_TIMEOUT, the awaited and the last seen value into status[0..2] (device
 * memory, nullable) and returns, so the stream never hangs. s8b_counter_add bumps an epoch
 * counter on the stream. s8b_flag_status reads status[0] from a host copy.              */
int s8b_flag_set(uint32_t *flag, const uint32_t *value, uint32_t add, void *stream);
int s8b_flag_wait(const uint32_t *flag, const uint32_t *value, uint32_t add,
                  uint64_t timeout_ns, int32_t *status, void *stream);
int s8b_counter_add(uint32_t *ctr, uint32_t inc, void *stream);
int s8b_flag_status(const int32_t *status_host_copy);
/* Copies n <= 8 buffers (bytes[i] from src[i] to dst[i], usually a peer's or an IPC-mapped
 * buffer) with plain stores from one CTA, then, if flag is not null, raises it exactly as
 * s8b_flag_set does, ordered after every copied byte. One launch instead of n copy-engine
 * copies and a flag launch: the hand-off of a sparse-MoE layer's token rows and routing to
 * a partner process holding other experts.                                                */
int s8b_peer_put_flag(void *const *dst, const void *const *src, const size_t *bytes, int n,
                      uint32_t *flag, const uint32_t *value, uint32_t add, void *stream);

/* Decode-step bookkeeping on the device: positions[i] += inc; context_lens[i] =
 * positions[i] + 1 (context_lens nullable). Keeps the per-step position state in device
 * memory so a captured step replays correctly (the reference rebuilds these tensors on the
 * host every step: superl8serve/dist/pipeline.py:1008-1009).                             */
int s8b_advance(int32_t *positions, int32_t *context_lens, int M, int inc, void *stream);

/* ---- set-up-time peer plumbing (not on the hot path) --------------------------------------
 * The reference moves boundary codes with tensor.to(dst) inside send()
 * (superl8serve/dist/__init__.py:214-247), which enables peer access implicitly. Here the
 * producer's encoder stores straight into the consumer's buffer, so peer access (one
 * process, several GPUs) or a CUDA IPC mapping (one process per GPU) is set up explicitly.
 * s8b_ipc_alloc is the only allocating entry point: it cudaMalloc's an exportable receive
 * buffer (zero-filled) and writes its s8b_ipc_handle_size()-byte handle to handle_out.      */
int s8b_enable_peer_access(int dev, int peer);
int s8b_ipc_handle_size(void);
int s8b_ipc_alloc(size_t bytes, void **ptr, void *handle_out);
int s8b_ipc_free(void *ptr);
int s8b_ipc_open(const void *handle, void **ptr);
int s8b_ipc_close(void *ptr);
/* One stream-ordered cudaMemcpyAsync (cudaMemcpyDefault) between device, peer, IPC-mapped or
 * pinned host addresses: host I/O around the step and set-up copies into raw buffers.      */
int s8b_memcpy_async(void *dst, const void *src, size_t bytes, void *stream);

/* ---- sparse-MoE FFN (Qwen3-MoE) -----------------------------------------------------
 * Replaces the router, the per-expert GatedMLP loop and the index_add_ combine of
 * SparseMoE.forward (superl8serve/models/moe.py:88-141; the experts' LinearW8A8 calls are
 * superl8.linear, superl8serve/layers/linear.py:122). A layer runs:
 *   s8b_moe_route(y)                        -> topi, topw, expert groups
 *   s8b_moe_gemm_grouped(xq, row=sorted_token, W_gate_up)  -> gu   [A, 2F] (A = T*top_k)
 *   s8b_silu_mul_quant(gu, A, F)            -> aq, as
 *   s8b_moe_gemm_grouped(aq, row=NULL, W_down)             -> part [A, H]
 *   s8b_moe_combine(part, topw, topi, assign_pos)          -> out  [T, H]
 *
 * s8b_moe_route: y [T, H] dtype (the post-attention RMSNorm output); gate [E, H] fp32
 * (16-byte aligned). Logits are float64 lane sums rounded to fp32, softmax over all E in
 * fp32 (exp_s8b), top_k largest (ties: lower expert first) in descending order,
 * renormalised by their sum (clamped at 1e-9) when norm_topk_prob, times routed_scaling,
 * rounded to dtype. Outputs: topi [T, top_k] int32, topw [T, top_k] dtype; the T*top_k
 * assignments a = t*top_k + j sorted by (expert, token): expert_offsets [E+1] (rows of
 * expert e are [off[e], off[e+1])), sorted_assign [A] (a at each sorted row),
 * sorted_token [A] (its token), assign_pos [A] (sorted row of each a).
 * H % 8 == 0, E <= 256, top_k <= min(16, E), T <= 4096. Two launches.                  */
int s8b_moe_route(const void *y, int dtype, const float *gate, int T, int H, int E, int top_k,
                  int norm_topk_prob, float routed_scaling, int32_t *topi, void *topw,
                  int32_t *expert_offsets, int32_t *sorted_assign, int32_t *sorted_token,
                  int32_t *assign_pos, void *stream);

/* Grouped W8A8 GEMM: for every expert e and row p in [expert_offsets[e], expert_offsets[e+1]),
 *   y[p, n] = dtype((float(sum_k xq[r, k] * w[e, n, k]) * xs[r]) * ws[e, n]),
 * r = row_index[p] (or p when row_index is NULL). w is int8 [E, N, K], ws fp32 [E, N];
 * A = expert_offsets[E] rows. K % 16 == 0, 40*K + 128 <= 200 KiB; xq, w 16-byte aligned.
 * Experts without rows cost nothing; every weight byte of a routed expert is read from HBM
 * once (staged in shared memory), whatever its row count.                                */
int s8b_moe_gemm_grouped(const int8_t *xq, const float *xs, const int32_t *row_index,
                         const int8_t *w, const float *ws, const int32_t *expert_offsets,
                         void *y, int A, int N, int K, int E, int dtype, void *stream);
/* The same grouped GEMM on the tensor cores (tcgen05 kind::i8, swap-AB: 128 weight rows of an
 * expert as M, the expert's rows as N), for the rows already in assignment order: xg [A, K]
 * int8 and xgs [A] (s8b_moe_gather_rows), so expert e's rows are xg[expert_offsets[e] ..
 * expert_offsets[e+1]). max_rows bounds every expert's row count (the token count: a token
 * routes to an expert at most once); experts with more than 64 rows take several passes.
 * Bit-identical to s8b_moe_gemm_grouped. K % 128 == 0, E <= 512, xg and w 16-byte aligned;
 * status: one int32 the caller zeroes, S8B_ERR_TIMEOUT after a bounded wait gave up.
 * Replaces the per-expert superl8.linear calls of SparseMoE.forward
 * (superl8serve/models/moe.py:135-141).                                                  */
int s8b_moe_gemm_grouped_tc(const int8_t *xg, const float *xgs, const int8_t *w, const float *ws,
                            const int32_t *expert_offsets, void *y, int A, int N, int K, int E,
                            int max_rows, int32_t *status, int dtype, void *stream);
/* Row gather into assignment order: xg[r] = xq[index[r]], xgs[r] = xs[index[r]], r < A.
 * K % 16 == 0. Feeds s8b_moe_gemm_grouped_tc. No counterpart in the reference.           */
int s8b_moe_gather_rows(const int8_t *xq, const float *xs, const int32_t *index, int A, int K,
                        int8_t *xg, float *xgs, void *stream);

/* out[t, :] = running dtype sum, in ascending expert index, of dtype(contrib[p, :] * w)
 * over the token's top_k assignments (p = assign_pos[t*top_k + j], w = topw[t, j]); each
 * product and each sum rounded to dtype, starting from zero (the reference's per-expert
 * out.index_add_). H % 4 == 0; contrib, out 8-byte aligned.                               */
int s8b_moe_combine(const void *contrib, const void *topw, const int32_t *topi,
                    const int32_t *assign_pos, void *out, int T, int top_k, int H, int dtype,
                    void *stream);

/* ---- rANS entropy stage --------------------------------------------------------------
 * Static byte-level rANS in the wire format of the reference's optional entropy stage
 * (superl8serve/dist/entropy.py encode / decode, called from superl8serve/dist/__init__.py:
 * 191-205, 279-288): frequencies freqs[256] normalised to sum 4096 (every symbol that occurs
 * >= 1), 32-bit state in [2^23, 2^31), symbols coded last to first, bytes emitted low byte
 * first, final state flushed as 4 bytes. The payload of n bytes is cut into n_streams
 * chunks (chunk i = [i*n/S, (i+1)*n/S)), each an independent stream coded by one GPU thread
 * into its own region at s8b_rans_stream_offset(n, S, i); with n_streams == 1 the region's
 * stream_len[0] bytes are exactly the reference's encode() output. 1 <= n_streams <= n. */
size_t s8b_rans_encoded_capacity(size_t n, int n_streams); /* 2n + 4*n_streams bytes    */
size_t s8b_rans_stream_offset(size_t n, int n_streams, int i);
/* counts[256] (uint32) = symbol histogram of sym[0..n) (zeroed here first).               */
int s8b_rans_histogram(const uint8_t *sym, size_t n, uint32_t *counts, void *stream);
/* stream_len[i] = bytes of stream i, or all ones if a symbol of chunk i has frequency 0.   */
int s8b_rans_encode(const uint8_t *sym, size_t n, const int32_t *freqs, int n_streams,
                    uint8_t *out, size_t out_capacity, uint64_t *stream_len, void *stream);
/* Decodes n symbols into out. Reads stay inside each stream's bytes; *bad = 1 if a stream
 * ends early (corrupt payload or wrong table). freqs must sum to 4096.                    */
int s8b_rans_decode(const uint8_t *enc, const uint64_t *stream_len, int n_streams,
                    const int32_t *freqs, size_t n, uint8_t *out, int32_t *bad, void *stream);

/* ---- sampler ------------------------------------------------------------------------
 * Replaces Sampler.forward (superl8serve/layers/sampler.py:22-86) for temperature, top_k,
 * top_p and repetition_penalty. Row r: x = f32(logits[r]); history[r][positions[r]] =
 * input_ids[r] is written first, then every distinct id of history[r][0..positions[r]]
 * gets x < 0 ? x*pen : x/pen; temperature 0 -> argmax (lowest index); otherwise
 * s = x / max(t, 1e-5), top_k > 0 keeps s >= the k-th largest, e = exp_s8b(s - max s),
 * q = floor(e * 2^32), top_p < 1 keeps every e whose strictly larger masses sum to
 * <= floor(p * sum q), and the token is the first index whose running sum of q exceeds
 * floor(u24 * Q * 2^-24), u24 = splitmix64(seeds[r] + positions[r]) >> 40. top_k, top_p and
 * penalty may be NULL (disabled). The reference draws torch-RNG Gumbel noise instead; the
 * distribution is the same categorical. workspace: s8b_sample_workspace_size(M, V) bytes.
 * V <= 2^24.                                                                            */
size_t s8b_sample_workspace_size(int M, int V);
int s8b_sample(const void *logits, int dtype, int M, int V, const float *temperature,
               const int32_t *top_k, const float *top_p, const float *penalty,
               const int32_t *input_ids, const int32_t *positions, int32_t *history,
               int history_cap, const uint64_t *seeds, void *workspace, size_t workspace_bytes,
               int32_t *out, void *stream);

/* ---- whole stage step ------------------------------------------------------------------
 * One decode (or prefill-chunk) step of one pipeline stage for one micro-batch of M rows,
 * enqueued on `stream` from a plain-pointer descriptor: the per-stage loop of
 * PipelineEngine._decode_microbatched (superl8serve/dist/pipeline.py:997-1040) over
 * Qwen3DecoderLayer.forward (superl8serve/models/qwen3.py:70-80), for hosts that drive the
 * library without Python. It launches exactly the kernels, in the same order, that the
 * Python stage runtime launches, so the two give identical results:
 *   [first] s8b_embed(ids) | [else] s8b_codec_decode(in_payload)
 *   per layer: rmsnorm_quant -> qkv GEMM -> qkv_post -> paged attention -> o GEMM ->
 *              rmsnorm_quant -> gate_up GEMM -> silu_mul_quant -> down GEMM
 *              (MoE layer: route -> grouped gate_up -> silu_mul_quant -> grouped down -> combine)
 *   [last]  rmsnorm_quant(final norm) -> head GEMM -> argmax | s8b_sample (writes ids)
 *   [else]  s8b_codec_encode(h, res) into out_payload (may be a peer's memory)
 * GEMMs run on the tensor cores (packed weight images) when tc_min > 0, M >= tc_min and a
 * packed image is given, with split-K partials in `part` between a GEMM and the row kernel
 * that follows it; otherwise on the dp4a path. Buffers are sized for M rows as the Python
 * runtime sizes them (StageRunner). Expert shards on other GPUs are not handled here.   */
typedef struct S8bLayerDesc {
  const int8_t *qkv_w, *qkv_packed; const float *qkv_s;
  const int8_t *o_w, *o_packed; const float *o_s;
  const int8_t *gu_w, *gu_packed; const float *gu_s; /* NULL in a sparse-MoE layer     */
  const int8_t *d_w, *d_packed; const float *d_s;
  const void *in_norm, *post_norm, *q_norm, *k_norm; /* gains, activation dtype        */
  int8_t *kc; float *ks; int8_t *vc; float *vs;      /* this layer's paged KV pool      */
  int moe_experts;                                   /* > 0: sparse-MoE FFN below       */
  int moe_top_k, moe_ffn, moe_norm_topk;
  float moe_scaling;
  const float *router;
  const int8_t *moe_gu_w; const float *moe_gu_s; const int8_t *moe_d_w; const float *moe_d_s;
} S8bLayerDesc;

typedef struct S8bStageDesc {
  int n_layers, M, H, Hq, Hkv, D, F, V;
  int block_size, max_blocks, max_ctx, rope_len, dtype, tc_min;
  int first_model_layer; /* 1: this stage's first layer is the model's layer 0            */
  int head;              /* last stage: 0 skips final norm / head / token choice           */
  float eps, scale;
  const S8bLayerDesc *layers;
  const float *cos_tab, *sin_tab;
  const void *embed;     /* first stage only                                               */
  const void *final_norm; const int8_t *head_w, *head_packed; const float *head_s; /* last */
  int32_t *ids, *positions, *context_lens, *block_table;
  const void *in_payload; const float *in_scales;  /* stages > 0                          */
  void *out_payload; float *out_scales;            /* all but the last stage              */
  int scheme;                                      /* S8B_CODEC_*                         */
  void *h, *res, *qkv, *attn, *gu, *logits;
  int8_t *xq; float *xs; int8_t *q_i8; float *q_s; int32_t *part;
  void *attn_ws; size_t attn_ws_bytes; void *tc_ws; size_t tc_ws_bytes;
  void *moe_y, *moe_topw, *moe_gu, *moe_contrib; int8_t *moe_aq; float *moe_as;
  int32_t *moe_topi, *moe_offsets, *moe_sorted_assign, *moe_sorted_token, *moe_assign_pos;
  /* sampling (temperature NULL: greedy argmax)                                           */
  const float *temperature, *top_p, *penalty; const int32_t *top_k;
  const int32_t *input_ids; int32_t *history; int history_cap; const uint64_t *seeds;
  void *sample_ws; size_t sample_ws_bytes;
} S8bStageDesc;

int s8b_stage_step(const S8bStageDesc *desc, void *stream);
/* sizeof of the two descriptors, for bindings that build them field by field */
size_t s8b_stage_desc_size(void);
size_t s8b_layer_desc_size(void);

#ifdef __cplusplus
}
#endif
#endif /* S8B_H_ */
