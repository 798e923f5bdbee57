/*
 * semantica_oracle.h — CPU restatement of go-semantica's embedding forward
 * pass and brute-force search, used ONLY as the test oracle and as the timed
 * CPU baseline. It is never linked into the product library.
 *
 * Parity status: partially pinned. The reference is Go and cannot be built on
 * this machine (no Go toolchain, no module cache, the GGUF weights are a
 * Git-LFS pointer), so this file restates the Go code operation by operation
 * (every function cites the reference file:line it follows) and is pinned by
 * the reference's own known-answer tests (prompt strings, softmax accuracy
 * bounds, Q8_0 scale round trips, brute dot-product tolerances, BRUT round
 * trips). The full 24-layer forward is not pinned against the running Go
 * binary: "parity unpinned" for the end-to-end embedding values.
 */
#ifndef SEMANTICA_ORACLE_H
#define SEMANTICA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar kernels (internal/kernels, internal/gguf) ---- */
float orc_f16_runtime(uint16_t h);                 /* internal/runtime/model_int8.go:571-597 */
float orc_f16_gguf(uint16_t h);                    /* internal/gguf/tensor.go:207-240 */
float orc_fast_exp(float x);                       /* internal/kernels/activation.go:100-145 */
void  orc_softmax(float *dst, const float *src, int n);            /* activation.go:161-213 */
void  orc_gelu_quick_simd(float *dst, const float *src, int n);    /* activation.go:47-95 */
float orc_dot_f32(const float *a, const float *b, int n);          /* simd_amd64.go:59-76, simd_amd64.s:19-76 */
void  orc_rmsnorm(float *dst, const float *src, const float *w, int n, float eps); /* norm.go:8-36 */
void  orc_quantize_sym_int8(const float *x, int64_t n, int8_t *codes, float *scale); /* quantize.go:29-103 */
void  orc_matmul_q8_0_int8(float *dst, const uint8_t *w_q8, const float *w_scales,
                           const int8_t *a, float a_scale, int batch, int in_dim, int out_dim);
                                                   /* quantize.go:346-458, simd_amd64.s:164-304 */
/* reference build to follow: 0 amd64 AVX512-VNNI (default), 1 amd64 AVX2, 2 portable noasm */
void  orc_set_matmul_path(int path);
int   orc_set_simd(int on); /* timing only: intrinsic inner loops, bit-identical results; returns 1 if on */
void  orc_extract_q8_0_scales(const uint8_t *w_q8, int64_t rows, int cols, float *scales);
                                                   /* model_int8.go:543-569 */

/* ---- model (internal/runtime) ---- */
typedef struct orc_model orc_model;

typedef struct {
    int32_t vocab_size, embed_dim, num_layers, num_heads, num_kv_heads, head_dim, interm_dim, max_seq_len;
    float norm_eps, rope_base, attention_scale;
} orc_config;

/* Opens a GGUF v3 file (internal/gguf/reader.go:33-178) and builds the model
 * exactly as internal/runtime/model.go:264-315 does. Returns NULL and writes
 * a message to err on failure. */
orc_model *orc_model_load(const char *path, char *err, int errlen);
void orc_model_free(orc_model *m);
void orc_model_config(const orc_model *m, orc_config *out);
/* Model-faithful mode (no reference counterpart): sliding-window layers (all
 * but every swa_pattern-th layer see keys within swa_window / 2 positions,
 * with RoPE base rope_base_swa when > 0) and the dense_2 / dense_3 head after
 * pooling. Zeros: the reference's forward. -1 if the head has no weights. */
int orc_model_set_faithful(orc_model *m, int swa_window, int swa_pattern, float rope_base_swa, int dense_head);

/* (*Model).ForwardWithDim (model.go:661-666 → model_int8.go:148-256) for ONE
 * sequence. Returns 0, or -1 with err set to the reference's message. */
int orc_forward(const orc_model *m, const int32_t *ids, int n, int target_dim,
                float *out, char *err, int errlen);

/* Many sequences, one per worker thread, as pkg/ggufembed/api.go:237-295 fans
 * out. out is packed: sequence s writes target_dim floats at out + s*target_dim.
 * nthreads <= 0 uses all cores. */
int orc_forward_batch(const orc_model *m, const int32_t *ids, const int32_t *offsets,
                      int nseq, int target_dim, float *out, int nthreads, char *err, int errlen);

/* ---- brute search (search/brute) ---- */
void  orc_normalize(float *v, int n);                                  /* builder.go:129-141 */
void  orc_quantize_int8_vec(const float *v, int n, int8_t *out);       /* quant.go:17-28 */
void  orc_quantize_int16_vec(const float *v, int n, int16_t *out);     /* quant.go:30-41 */
float orc_dot_int8_ref(const int8_t *v, const float *q, int dim);      /* quant.go:83-108, dot_amd64.s:12-43 */
float orc_dot_int16_ref(const int16_t *v, const float *q, int dim);    /* quant.go:110-135, dot_amd64.s:46-77 */
float orc_dot_f32_ref(const float *a, const float *b, int dim);        /* index.go:198-214, dot_amd64.s:80-105 */

/* index.go:55-154 verbatim (fp32 query, running min-replace top-k, final sort
 * by (distance desc, id asc)). quant: 0 f32, 1 int8, 2 int16. Returns the
 * number of results written. */
int orc_search_ref(int quant, const void *data, const int32_t *ids, int64_t count, int dim,
                   const float *query_normalized, int topk, int32_t *out_ids, float *out_dist);

/* Integer contract: query quantised like the stored rows (quant.go:17-41),
 * score = sum int32(q)*int32(v) exactly, top-k by (score desc, row asc),
 * distance = score / scale^2 (double division, rounded to float). quant 1 or 2.
 * Fills out_rows (row positions), out_scores; returns the number of results. */
int orc_search_exact(int quant, const void *data, int64_t count, int dim,
                     const void *query_codes, int topk, int32_t *out_rows, int32_t *out_scores,
                     float *out_dist);
int orc_search_exact_batch(int quant, const void *data, int64_t count, int dim,
                           const void *query_codes, int nq, int topk, int32_t *out_rows,
                           int32_t *out_scores, float *out_dist, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
