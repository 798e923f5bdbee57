/*
 * semantica_b200.h — C ABI of libsemantica_b200.so, the B200 (sm_100a)
 * implementation of go-semantica's two data-parallel hot paths:
 *
 *   1. the EmbeddingGemma INT8 forward pass behind rt.Embed
 *      (internal/runtime.(*Model).ForwardWithDim, model.go:661-666), and
 *   2. search/brute's quantised scan + top-k behind Index.SearchVector and
 *      the BRUT v1 Serializer (search/brute/index.go, storage.go).
 *
 * Plain C types only: pointers, sizes, status codes. Every call returns a
 * SEM_* status; on failure sem_last_error() returns a message that matches the
 * reference's error string where the reference has one. No call keeps a
 * pointer to caller memory after it returns (the cgo rule): inputs are copied.
 * A context is bound to one GPU; calls on one context are serialised.
 *
 * Citations are "file:line" inside the go-semantica source tree.
 */
#ifndef SEMANTICA_B200_H
#define SEMANTICA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define SEM_OK 0
#define SEM_EINVAL 1    /* invalid argument (reference-style message in sem_last_error) */
#define SEM_EDEVICE 2   /* CUDA error */
#define SEM_ENOMEM 3    /* device or host allocation failed */
#define SEM_EFORMAT 4   /* malformed GGUF or BRUT bytes */
#define SEM_ENOTFOUND 5 /* tensor / id not found */
#define SEM_EINTERNAL 6 /* a host-side failure inside the library (e.g. a thread could not start) */

typedef struct sem_context sem_context;
typedef struct sem_model sem_model;
typedef struct sem_index sem_index;
typedef struct sem_q8_weight sem_q8_weight;
typedef struct sem_group sem_group;

/* Message of the last failed call on this thread (never NULL). A Go caller
 * holds its OS thread (runtime.LockOSThread) from the failing call until it
 * has read the message: a goroutine may change threads between cgo calls. */
const char *sem_last_error(void);

/* Number of visible CUDA devices. */
int sem_device_count(int *out);

/* A context owns one device, one stream and the device workspaces. */
int sem_context_create(int device, sem_context **out);
int sem_context_destroy(sem_context *ctx);
/* The context's CUDA stream, as a cudaStream_t. */
void *sem_context_stream(sem_context *ctx);

/* ------------------------------------------------------------------------
 * Model: replaces internal/runtime.LoadModel / loadModel (model.go:233-315)
 * ---------------------------------------------------------------------- */

/* Mirrors internal/runtime.ModelConfig (model.go:16-31). */
typedef struct sem_model_config {
  int32_t vocab_size, embed_dim, num_layers, num_heads, num_kv_heads, head_dim, interm_dim, max_seq_len;
  float norm_eps, rope_base, attention_scale;
} sem_model_config;

/* A GGUF tensor as internal/gguf.Reader exposes it (reader.go:23-30,
 * :332-346): dims are GGUF ne[] (ne0 contiguous), dtype is the GGUF type id
 * (0 F32, 8 Q8_0), data points at the tensor bytes (e.g. into the mmap). */
typedef struct sem_tensor_view {
  const char *name;
  uint32_t dtype;
  uint32_t n_dims;
  uint64_t dims[4];
  const void *data;
  uint64_t nbytes;
} sem_tensor_view;

/* Uploads the model named by `tensors` (token_embd.weight, output_norm.weight,
 * blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,attn_q_norm,attn_k_norm,
 * post_attention_norm,ffn_norm,ffn_gate,ffn_up,ffn_down,post_ffw_norm}.weight,
 * model_int8.go:54-119) to the context's device, repacking every Q8_0 tensor
 * into an int8 plane and an fp32 block-scale plane. The caller's bytes may be
 * released when the call returns. Replaces loadWeights + loadLayerINT8
 * (model.go:520-552, model_int8.go:54-119). */
int sem_model_load(sem_context *ctx, const sem_model_config *cfg, const sem_tensor_view *tensors, int32_t n_tensors,
                   sem_model **out);

/* Convenience: parses a GGUF v3 file the way internal/gguf + parseConfig do
 * (reader.go:98-178, model.go:424-517) and calls sem_model_load. */
int sem_model_load_gguf(sem_context *ctx, const char *path, sem_model **out);

int sem_model_config_get(const sem_model *model, sem_model_config *out);
int sem_model_free(sem_model *model);

/* ------------------------------------------------------------------------
 * Embedding forward: replaces (*Model).ForwardWithDim (model.go:661-666 →
 * model_int8.go:148-256), batched. The reference runs one sequence per call
 * and fans calls out over goroutines (pkg/ggufembed/api.go:237-295); here one
 * call carries every sequence of a request.
 * ---------------------------------------------------------------------- */

/* ids: packed token ids of n_seqs sequences; offsets: n_seqs+1 prefix offsets
 * into ids; dims: per-sequence output dimension (1..embed_dim; NULL = embed_dim
 * for all); out: packed outputs, sequence s at sum(dims[0..s-1]), each the
 * mean-pooled, L2-normalised first dims[s] channels.
 * Errors (reference strings): "empty input", "sequence too long: %d > %d",
 * "token ID out of range: %d", "target dimension %d out of range (1..%d)". */
int sem_embed(sem_model *model, const int32_t *ids, const int32_t *offsets, int32_t n_seqs, const int32_t *dims,
              float *out);

/* Device-resident variant (no host copies): d_ids on the device, h_offsets on
 * the host, d_out on the device (n_seqs x dim). Enqueued on `stream` (NULL =
 * the context stream); returns without synchronising, so errors the device
 * detects (a token id outside the vocabulary, a timed-out pipeline wait)
 * surface through sem_model_check. */
int sem_embed_device(sem_model *model, const int32_t *d_ids, const int32_t *h_offsets, int32_t n_seqs, int32_t dim,
                     float *d_out, void *stream);

/* The request pipeline (no reference counterpart; it stands in for the
 * reference's one goroutine per prompt, pkg/ggufembed/api.go:237-295, at the
 * level of whole requests). sem_embed_submit checks a request exactly as
 * sem_embed does, copies its ids and metadata into one of the model's two
 * request slots (pinned host staging), enqueues the upload, the forward and
 * the download of its outputs, and returns a ticket without waiting.
 * sem_embed_wait(ticket) blocks until that request is done and writes its
 * outputs (sem_embed's layout) to `out`. While one request runs on the
 * device the host prepares (tokenises, submits) the next. At most two
 * requests are in flight: a third submit fails with SEM_EINVAL until one is
 * waited for. Requests run in submission order; each ticket is waited for
 * once. Errors the device reports (a timed-out pipeline wait) are returned by
 * sem_embed_wait. */
int sem_embed_submit(sem_model *model, const int32_t *ids, const int32_t *offsets, int32_t n_seqs,
                     const int32_t *dims, uint64_t *ticket);
int sem_embed_wait(sem_model *model, uint64_t ticket, float *out);

/* Waits for the model's device to finish every forward enqueued so far and
 * reports what the device recorded since the last check (or sem_embed call):
 * SEM_EINVAL "token ID out of range: ..." for a device-resident id outside the
 * vocabulary (its embedding row was written as zeros), SEM_EDEVICE when a
 * tensor-core pipeline wait timed out (that kernel returned early and its
 * output is incomplete). Clears the record. No reference counterpart: the
 * reference validates ids on the host (model_int8.go:167-178). */
int sem_model_check(sem_model *model);

/* Model-faithful mode. The reference runs full bidirectional attention in
 * every layer and has no dense head (model_int8.go:235-255, :500); the
 * EmbeddingGemma architecture has both, and this mode restores them. It has
 * no counterpart in the reference and is off by default (sem_embed computes
 * the reference's forward).
 *   sliding_window: in sliding layers query i sees keys j with
 *     |i - j| <= sliding_window / 2 (0: every layer sees every key);
 *   swa_pattern: layer l (0-based) is a global layer when (l + 1) % swa_pattern
 *     == 0, a sliding layer otherwise (EmbeddingGemma: window 512, pattern 6);
 *   rope_base_swa: RoPE base of the sliding layers (0: the model's rope_base);
 *   dense_head: after output_norm and mean pooling of every channel, the
 *     dense_2.weight (embed -> mid) and dense_3.weight (mid -> embed) Q8_0
 *     projections, each input quantised per sequence like every projection of
 *     the forward; then the first dims[s] outputs, L2-normalised. The weights
 *     are read at load when the tensors are present. */
typedef struct sem_faithful_config {
  int32_t sliding_window, swa_pattern;
  float rope_base_swa;
  int32_t dense_head;
} sem_faithful_config;
/* cfg NULL (or all zero): the reference's forward. Errors: SEM_EINVAL for
 * negative fields or a dense head the model has no weights for. */
int sem_model_set_faithful(sem_model *model, const sem_faithful_config *cfg);

/* ------------------------------------------------------------------------
 * Several GPUs of one host as one embedding engine. The reference fans the
 * sequences of a request out over goroutines (pkg/ggufembed/api.go:237-295);
 * a group fans them out over devices: one context and one model replica per
 * device, each request split by token count (longest sequence first to the
 * device holding the fewest tokens) and embedded on every device at once from
 * one host thread per device. No collective: replicas share nothing.
 * ---------------------------------------------------------------------- */

/* Loads the model on each of the n_devices distinct devices (in parallel). */
int sem_group_load(const int32_t *devices, int32_t n_devices, const sem_model_config *cfg,
                   const sem_tensor_view *tensors, int32_t n_tensors, sem_group **out);
int sem_group_load_gguf(const int32_t *devices, int32_t n_devices, const char *path, sem_group **out);
int sem_group_size(const sem_group *group, int32_t *out);
int sem_group_config_get(const sem_group *group, sem_model_config *out);
/* sem_model_set_faithful on every replica, or on none: when one replica fails,
 * those already switched return to their previous setting and the error names
 * the device. */
int sem_group_set_faithful(sem_group *group, const sem_faithful_config *cfg);
/* sem_embed's contract (same arguments, errors and output layout); the
 * request is validated on the host before any device starts, and a device's
 * error is returned as "device N: <message>". One request at a time per
 * group; concurrent callers wait. */
int sem_group_embed(sem_group *group, const int32_t *ids, const int32_t *offsets, int32_t n_seqs,
                    const int32_t *dims, float *out);
int sem_group_free(sem_group *group);

/* Per-stage device timing of the forward pass (diagnostics; no reference
 * counterpart). enable != 0 brackets every kernel launch of later forwards
 * with CUDA events on the launching stream. profile_read synchronises the
 * context stream, returns up to `cap` stages (static names, total ms, launch
 * counts) accumulated since the last read, and resets the totals. */
int sem_model_profile(sem_model *model, int32_t enable);
int sem_model_profile_read(sem_model *model, const char **names, float *total_ms, int32_t *launches, int32_t cap,
                           int32_t *n_out);

/* ------------------------------------------------------------------------
 * Isolated Q8_0 x INT8 projection: QuantizeSymmetricINT8Into + MatMulQ8_0INT8
 * (internal/kernels/quantize.go:29-69, :346-458).
 * ---------------------------------------------------------------------- */

/* w_q8: raw Q8_0 bytes of an [n_out rows x k_in] weight (GGUF dims {k_in, n_out}). */
int sem_q8_weight_create(sem_context *ctx, const void *w_q8, int32_t k_in, int32_t n_out, sem_q8_weight **out);
int sem_q8_weight_free(sem_q8_weight *w);
/* Device pointers: d_a fp32 [m x k_in] -> d_c fp32 [m x n_out], one activation
 * scale for the whole of d_a as in the reference; d_codes and d_absmax (one
 * uint32) are caller-provided scratch. d_codes holds the m x k_in INT8 codes
 * as fp16 (the tensor cores' operand type; 2 * m * k_in bytes, 16-byte
 * aligned). Enqueued on `stream`. */
int sem_q8_gemm(sem_q8_weight *w, const float *d_a, int32_t m, float *d_c, void *d_codes, uint32_t *d_absmax,
                void *stream);

/* MatMulQ8_0INT8 alone (quantize.go:346-458) on activations already quantised
 * by QuantizeSymmetricINT8Into: d_codes holds the m x k_in INT8 codes as fp16
 * (16-byte aligned), *d_absmax the float32 bit pattern of the absmax they were
 * quantised with (scale = absmax / 127, as quantize.go:60-61); d_c fp32
 * [m x n_out]. Enqueued on `stream`. */
int sem_q8_matmul_int8(sem_q8_weight *w, const void *d_codes, const uint32_t *d_absmax, int32_t m, float *d_c,
                       void *stream);

/* Which kernel the Q8_0 projections use (process-wide, every model and
 * weight). Three kernels exist:
 *   - the CUDA-core kernel computes the reference's VNNI inner loop exactly
 *     (simd_amd64.s:241-304: 8 float32 lane accumulators, each a fused
 *     multiply-add of an exact 4-product int32 partial and the block scale,
 *     then the reference's horizontal sum and the unfused inputScale
 *     multiply): bit-identical to the reference's default amd64 build;
 *   - the per-block tensor-core kernel sums each 32-element block exactly and
 *     scales it in float32, accumulating the blocks in another order;
 *   - the split-plane tensor-core kernel folds the block scales into two fp16
 *     weight planes (one TMEM drain per tile, the fastest at scale) and differs
 *     from the reference's sums in the last float32 bits.
 * sem_embed packs sequences of >= 128 tokens first. Shorter sequences (while
 * a batch holds at most 4096 of their tokens; beyond that they take the
 * tensor-core kernels as long rows do) take the CUDA-core kernel (and a
 * float32 attention in the reference's order), so their embeddings are
 * bit-identical to the reference's; long-sequence rows
 * take a tensor-core kernel (mean pooling over many tokens keeps the
 * difference within the reference's own spread between its builds).
 *   SEM_Q8_PATH_AUTO (default): long-sequence rows take the split-plane kernel
 *     when its 128 x 256-token tiles fill at least half the SMs, else the
 *     per-block kernel; sem_q8_gemm / sem_q8_matmul_int8 take the CUDA-core
 *     kernel below 128 rows, then the same rule;
 *   SEM_Q8_PATH_BLOCK: the per-block kernel everywhere;
 *   SEM_Q8_PATH_SPLIT: the split-plane kernel for long-sequence rows (all
 *     rows for sem_q8_gemm) whatever their count;
 *   SEM_Q8_PATH_SPLIT_ALL: the split-plane kernel for every row (testing);
 *   SEM_Q8_PATH_EXACT: the CUDA-core kernel for every row (bit-exact
 *     projections at any length, slower than the tensor cores at scale).
 * A tuning and testing switch with no counterpart in the reference. Returns
 * the previous setting, or -1 for an unknown mode. */
#define SEM_Q8_PATH_AUTO 0
#define SEM_Q8_PATH_BLOCK 1
#define SEM_Q8_PATH_SPLIT 2
#define SEM_Q8_PATH_SPLIT_ALL 3
#define SEM_Q8_PATH_EXACT 4
int sem_q8_path(int32_t mode);

/* sem_q8_gemm without caller scratch, for callers that cannot allocate device
 * memory (a host runtime that owns the whole device pool and passes only input
 * and output buffers, or a request path with a memory budget fixed at start-up
 * where an allocation may neither grow nor fail). It has no counterpart in the
 * reference. The codes and the absmax word live in a static device array of
 * 16 MiB + 256 bytes that every GPU loading the library holds until exit, so
 * m * k_in must not exceed 8 Mi (8,388,608) elements (larger calls fail with
 * SEM_EINVAL); m == 0 is a no-op, as for sem_q8_gemm. The kernel choice is
 * sem_q8_gemm's (sem_q8_path). The call performs no allocation. The first
 * call on a device resolves the array's address on that device
 * (cudaGetSymbolAddress), which loads the library's device code there and may
 * synchronise the device; the array's 16 MiB are committed then, not when the
 * library is loaded. Make that first call (a warm-up call will do) at start-up,
 * before the host runtime reserves its device pool and before any stream
 * capture. All calls share the one array: calls that overlap on the GPU (other
 * streams, other threads) race on it. Enqueued on `stream` (NULL = the
 * weight's context stream). */
int sem_q8_gemm_noalloc(sem_q8_weight *w, const float *d_a, int32_t m, float *d_c, void *stream);

/* ------------------------------------------------------------------------
 * Brute-force index: replaces search/brute (builder.go, index.go, storage.go).
 * quant: 0 float32, 1 int8, 2 int16 (brute.QuantizationMode, quant.go:8-15).
 * ---------------------------------------------------------------------- */

/* Builder.AddVector + Build (builder.go:52-127): vectors are normalised
 * (builder.go:129-141) and quantised (quant.go:17-41) on the device.
 * ids must be unique ("brute: duplicate id %d"). */
int sem_index_build(sem_context *ctx, int32_t dim, int32_t quant, const float *vectors, const int32_t *ids,
                    int64_t count, sem_index **out);

/* An index from already-stored rows (codes as Build or Deserialize produce
 * them): data is count x dim of int8 / int16 / float32, in host or device
 * memory. int8 indexes with dim >= 128 search on the tensor cores. */
int sem_index_create(sem_context *ctx, int32_t dim, int32_t quant, const void *data, const int32_t *ids, int64_t count,
                     sem_index **out);

int sem_index_free(sem_index *idx);
int sem_index_count(const sem_index *idx, int64_t *out);
int sem_index_dimension(const sem_index *idx, int32_t *out);
int sem_index_quantization(const sem_index *idx, int32_t *out);

#define SEM_SEARCH_REFERENCE 0 /* fp32 query x (code/127): the reference's own arithmetic */
#define SEM_SEARCH_EXACT 1     /* query quantised like the rows, exact int32 dot products */

/* Index.SearchVector (index.go:29-42) for nq queries (nq x dim floats, not
 * yet normalised; normalize != 0 normalises them first as SearchVector does,
 * 0 treats them as normalised like SearchNormalized, :44-53). Results per
 * query: min(k, count) entries, best first; ties break toward the lower row.
 * out_ids/out_dist are nq x k (unused tail entries: id -1). out_scores (exact
 * mode, may be NULL) receives the int32 scores. Errors: "brute: topK must be
 * positive", "brute: query dimension mismatch: got %d want %d". */
int sem_index_search(sem_index *idx, const float *queries, int32_t nq, int32_t dim, int32_t k, int32_t mode,
                     int32_t normalize, int32_t *out_ids, float *out_dist, int32_t *out_scores);

/* Device-level search of one shard for multi-GPU merges: d_qcodes (exact
 * mode, nq x dim codes of the index's element type) or d_queries (reference
 * mode, normalised floats); writes nq x k 64-bit candidate keys
 * ((order-preserving score << 32) | ~global_row) to d_keys, where global_row =
 * row_base + local row. Enqueued on `stream`. */
int sem_index_search_keys(sem_index *idx, const void *d_queries, int32_t nq, int32_t k, int32_t mode,
                          int64_t row_base, uint64_t *d_keys, void *stream);

/* Merges `lists` candidate-key lists of k per query (d_keys: lists x nq x k)
 * into the best k_out per query. quant selects the distance scale (1: /127^2,
 * 2: /32767^2) for exact-mode keys. Any output may be NULL. */
int sem_topk_merge(sem_context *ctx, const uint64_t *d_keys, int32_t lists, int32_t nq, int32_t k, int32_t k_out,
                   int32_t mode, int32_t quant, int32_t *d_rows, int32_t *d_scores, float *d_dist, void *stream);

/* Quantises normalised queries exactly like stored rows (quant.go:17-41). */
int sem_quantize_queries(const float *queries, int32_t nq, int32_t dim, int32_t quant, void *out_codes);

/* Index.Vector (index.go:162-180): dequantised copy of the row with this id. */
int sem_index_vector(sem_index *idx, int32_t id, float *out);

/* BRUT v1 (storage.go:17-153): 20-byte header {"BRUT", u16 version 1, u16 dim,
 * u32 count, u8 quantization, 7 pad}, int32 ids[count], row-major data; little
 * endian. serialize: pass buf = NULL to get the size in *written. */
int sem_index_serialize(sem_index *idx, void *buf, size_t cap, size_t *written);
int sem_index_deserialize(sem_context *ctx, const void *bytes, size_t n, sem_index **out);

#ifdef __cplusplus
}
#endif
#endif
