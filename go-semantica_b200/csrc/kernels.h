// Host-side launch wrappers for the sm_100a kernels. Plain pointers and sizes
// only; every wrapper enqueues on `stream` and returns the launch status.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sem {

// ---- load-time repacking (model_kernels.cu) ----
// Q8_0 blocks (fp16 scale + 32 int8, 34 bytes) of `rows` x `cols` -> an int8
// plane (dst_codes[dst_row][cols]) and an fp32 scale plane
// (dst_scales[dst_row][cols/32]). f16 decoding follows the reference's
// runtime decoder (gguf_decoder = false, model_int8.go:571-597) or its gguf
// decoder (true, gguf/tensor.go:207-240). Row r goes to dst_row_offset + map(r),
// where map interleaves groups of `interleave` rows with a partner tensor
// (part 0 or 1) when interleave > 0.
cudaError_t launch_repack_q8_0(const uint8_t* raw, int64_t rows, int cols, int8_t* dst_codes,
                               float* dst_scales, int64_t dst_row_offset, int interleave, int part,
                               bool gguf_decoder, cudaStream_t stream);

// Projection weights for the tensor-core GEMM: Q8_0 blocks of `rows` x `cols`
// -> fp16 codes (exact integers) dst_codes[dst_row_offset + r][cols] and fp32
// block scales dst_scales[dst_row_offset + r][cols/32] (runtime f16 decoder,
// model_int8.go:571-597).
cudaError_t launch_repack_q8_0_f16(const uint8_t* raw, int64_t rows, int cols, __half* dst_codes,
                                   float* dst_scales, int64_t dst_row_offset, cudaStream_t stream);

// Projection weights for the split-plane GEMM: Q8_0 blocks of `rows` x `cols`
// -> fp16 planes hi/lo [dst_row_offset + r][cols] with hi + lo = q * d * 2^S_r
// and row_scale[dst_row_offset + r] = 2^-S_r (runtime f16 decoder).
cudaError_t launch_repack_q8_0_split(const uint8_t* raw, int64_t rows, int cols, __half* hi, __half* lo,
                                     float* row_scale, int64_t dst_row_offset, cudaStream_t stream);

// ---- forward-pass element-wise kernels (model_kernels.cu) ----
struct SeqMeta {
  const int32_t* row_seq;   // [T] sequence of each packed row
  const int32_t* row_pos;   // [T] position of each row within its sequence
  const int32_t* cu_seqlens;// [B+1]
  int32_t T;                // rows
  int32_t B;                // sequences
};

// Where a QKV projection may put its V columns: [col0, col0 + 256) of each
// row as the attention's fp16 hi and lo planes (hi[row][256], lo = hi + rows
// * 256) instead of the float32 output. Only the split-plane kernel does so;
// launch_q8_proj sets *written to whether this call did.
struct VPlanes {
  __half* hi = nullptr;
  int64_t rows = 0;
  int col0 = 0;
  bool* written = nullptr;
};

cudaError_t launch_embed(const int32_t* ids, const int8_t* emb_codes, const float* emb_scales, int vocab,
                         int H, float* hidden, int T, uint32_t* err_flag, cudaStream_t stream);

// inv_rms[row] of hidden rows with the norm weight w, and atomically the
// per-sequence absmax of the normed rows into absmax[seq] (absmax may be null).
cudaError_t launch_row_stats(const float* x, const float* w, int H, float eps, SeqMeta meta, float* inv_rms,
                             uint32_t* absmax, cudaStream_t stream);

// codes = quantize((x * inv_rms[row]) * w) with the per-sequence scale; when
// inv_rms is null the rows are quantized as they are; a null meta.row_seq
// means one scale (absmax[0]) for every row. The INT8 codes are stored as
// fp16 (exact), the tensor-core GEMM's operand type.
cudaError_t launch_quantize(const float* x, const float* inv_rms, const float* w, int K, SeqMeta meta,
                            const uint32_t* absmax, __half* codes, cudaStream_t stream);

// dst[i] = src[idx[i]] for i < n (packing token ids in the forward's order).
cudaError_t launch_gather_i32(const int32_t* src, const int32_t* idx, int32_t* dst, int64_t n, cudaStream_t stream);

// Max |x| over n values, atomically into slot[0].
cudaError_t launch_absmax(const float* x, int64_t n, uint32_t* slot, cudaStream_t stream);

// Per-head RMSNorm of q (num_heads heads) and k (1 head), NeoX RoPE, and the
// hi/lo fp16 split of q, k, v for attention. qkv rows: [q (nh*256) | k (256) | v (256)].
// Rows >= f32_row0 also get their normed, RoPE'd q and k written back into qkv
// as float32 (the input of launch_attention_short).
// Rows below v_row0 have their V planes already (written by the projection).
cudaError_t launch_qk_norm_rope(float* qkv, const float* q_norm, const float* k_norm, const float* rope_cos,
                                const float* rope_sin, float eps, int num_heads, SeqMeta meta, __half* qh,
                                __half* ql, __half* kh, __half* kl, __half* vh, __half* vl, int64_t f32_row0,
                                int64_t v_row0, cudaStream_t stream);

// hidden = rmsnorm(o, post_w) + hidden and inv_rms of the new rows for the
// next norm (next_w); with codes (and absmax) also the next norm's output
// quantized with its per-sequence scale: absmax[seq] = max |(hidden *
// inv_rms) * next_w| over the sequence, codes as in launch_quantize. codes and
// absmax are both null or both set. H is 256, 512 or 768; meta.cu_seqlens is
// required (a cluster of CTAs owns one sequence at a time).
cudaError_t launch_residual_norm(const float* o, const float* post_w, float* hidden, const float* next_w, int H,
                                 float eps, SeqMeta meta, float* inv_rms, uint32_t* absmax, __half* codes,
                                 cudaStream_t stream);

// Mean pooling of the first out_dim[s] columns of (hidden * inv_rms) * w over
// each sequence, then L2 normalisation; writes out + out_offset[s]. With
// out_dims null: every column, no normalisation, sequence s at out + s * H.
cudaError_t launch_pool_l2(const float* hidden, const float* inv_rms, const float* w, int H, SeqMeta meta,
                           const int32_t* out_dims, const int64_t* out_offsets, float* out, cudaStream_t stream);

// Each of `rows` rows of K floats quantised as its own INT8 buffer
// (QuantizeSymmetricINT8Into, quantize.go:29-69): absmax bit pattern into
// absmax[row], codes (held as fp16) into codes[row][K]. K % 4 == 0.
cudaError_t launch_quantize_rows(const float* x, int rows, int K, uint32_t* absmax, __half* codes,
                                 cudaStream_t stream);
// l2Normalize (model.go:808-820) of the first out_dims[r] values of each row
// of x ([rows][K]) into out + out_offsets[r].
cudaError_t launch_l2_rows(const float* x, int rows, int K, const int32_t* out_dims, const int64_t* out_offsets,
                           float* out, cudaStream_t stream);

// ---- Q8_0 x INT8 projection (gemm_q8.cu) ----
enum GemmEpilogue { kEpiStore = 0, kEpiGeluUp = 1 };
// C[m, n] = in_scale[seq(m)] * sum_kb float(exact block dot) * w_scales[n, kb].
// a_codes: fp16 INT8 codes [M][K]; w_codes: fp16 codes [N][K]; w_scales fp32
// [N][K/32]; all 16-byte aligned, K % 128 == 0, N % 128 == 0. kEpiGeluUp: rows [0, N/2) are gate and
// [N/2, N) up (N/2 % 128 == 0); writes h[m, n] = gelu_quick(gate) * up for
// n < N/2 and the per-sequence absmax of h. `err` (nullable) receives error
// bits if a pipeline wait times out.
cudaError_t launch_gemm_q8(const __half* a_codes, const __half* w_codes, const float* w_scales, int M, int N,
                           int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c, int epilogue,
                           uint32_t* out_absmax, uint32_t* err, cudaStream_t stream);

// The same product with the block scales folded into split fp16 weight planes
// (gemm_split.cu): w_hi/w_lo [N][K], row_scale [N]; K % 64 == 0, N % 128 == 0
// (gate/up: N/2 % 128 == 0). Same epilogues and outputs as launch_gemm_q8.
cudaError_t launch_gemm_q8_split(const __half* a_codes, const __half* w_hi, const __half* w_lo, const float* row_scale,
                                 int M, int N, int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c,
                                 int epilogue, uint32_t* out_absmax, uint32_t* err, cudaStream_t stream,
                                 const VPlanes& vp = VPlanes{});

// The same product on CUDA cores in the reference's VNNI lane order
// (gemm_dp4a.cu): bit-identical to matmulInnerLoopVNNIAsm + the unfused
// inputScale multiply. w_lanes: the int8 plane [N][K] with each row stored
// lane-major (launch_repack_q8_0_lanes); w_scales: fp32 block scales
// [N][K/32]; K % 128 == 0, N % 128 == 0. Same epilogues and outputs as
// launch_gemm_q8.
cudaError_t launch_gemm_q8_dp4a(const __half* a_codes, const int8_t* w_lanes, const float* w_scales, int M, int N,
                                int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c, int epilogue,
                                uint32_t* out_absmax, cudaStream_t stream);
// Q8_0 blocks of `rows` x `cols` -> the lane-major int8 plane of
// launch_gemm_q8_dp4a: row dst_row_offset + r, 32-bit word (lane * cols/32 +
// block) = bytes 4 lane .. 4 lane + 3 of that block.
cudaError_t launch_repack_q8_0_lanes(const uint8_t* raw, int64_t rows, int cols, int8_t* dst, int64_t dst_row_offset,
                                     cudaStream_t stream);

// A Q8_0 projection weight [N][K] in its device layouts: fp16 codes with fp32
// block scales (launch_gemm_q8), the split planes (launch_gemm_q8_split) and
// the lane-major int8 plane (launch_gemm_q8_dp4a, with the same block scales).
struct Q8Proj {
  const __half* codes;     // [N][K]
  const float* scales;     // [N][K/32]
  const __half* hi;        // [N][K]
  const __half* lo;        // [N][K]
  const float* row_scale;  // [N]
  const int8_t* lanes;     // [N][K], lane-major rows
};
// Picks the kernel for M tokens: the CUDA-core VNNI-order kernel below
// kDp4aMaxRows rows, the split-plane GEMM once its tiles fill half the SMs
// (measured crossover), else the per-block kernel (narrower token tiles, half
// the weight bytes). sem_q8_path overrides the choice.
constexpr int kDp4aMaxRows = 128;
cudaError_t launch_q8_proj(const __half* a_codes, const Q8Proj& w, int M, int N, int K, const uint32_t* a_absmax,
                           const int32_t* row_seq, float* c, int epilogue, uint32_t* out_absmax, uint32_t* err,
                           cudaStream_t stream, const VPlanes& vp = VPlanes{});
// Process-wide kernel choice: 0 auto, 1 per-block, 2 split-plane (launch_q8_proj
// always; the forward's long-sequence rows), 3 split-plane for every forward
// row, 4 the CUDA-core VNNI-order kernel for every row; returns the previous
// one (-1: unknown mode, nothing changed).
int set_q8_path(int mode);
int get_q8_path();

// ---- attention (attention.cu) ----
constexpr int kAttnTileRows = 128;  // query rows per attention tile
struct AttnTiles {
  const int32_t* tile_seq;    // [n_tiles] sequence of each 128-query tile
  const int32_t* tile_row0;   // [n_tiles] first packed row of the tile
  int32_t n_tiles;
};
// q planes [T][num_heads][256], k and v planes [T][256] (fp16 hi/lo splits;
// kl == kh + T * 256 and vl == vh + T * 256: the lo planes follow the hi ones),
// all 16-byte aligned. out [T][num_heads*256] fp32, absmax[seq] atomically.
// half_window > 0: a sliding-window layer, query i sees keys j with
// |i - j| <= half_window (0: every key). Full attention with pair_tiles (256-
// row query tiles: tile_row0 and tile_row0 + 128, n_tiles > 0) runs on SM
// pairs; otherwise one CTA per 128-row tile of `tiles`. `err` (nullable)
// receives error bits if a pipeline wait times out.
cudaError_t launch_attention(const __half* qh, const __half* ql, const __half* kh, const __half* kl,
                             const __half* vh, const __half* vl, int num_heads, float scale, int half_window,
                             SeqMeta meta, AttnTiles tiles, AttnTiles pair_tiles, float* out, uint32_t* absmax,
                             uint32_t* err, cudaStream_t stream);

// Float32 attention of sequences shorter than 128 tokens in the reference's
// order (attention_short.cu): qkv rows [q (nh*256) | k | v] float32 with q and
// k normed and RoPE'd (launch_qk_norm_rope with f32_row0 at or below their
// rows); `tiles` lists one 128-row tile per such sequence, max_len is the
// longest of them (at most 127). half_window as launch_attention. out
// [T][nh*256], absmax[seq] atomically, as launch_attention.
cudaError_t launch_attention_short(const float* qkv, int num_heads, float scale, int half_window, SeqMeta meta,
                                   AttnTiles tiles, int max_len, float* out, uint32_t* absmax, cudaStream_t stream);

// ---- brute search (brute_kernels.cu) ----
// Exact integer scan: scores of nq queries against rows [0, count) of an
// int8 (elem 1) or int16 (elem 2) corpus; per-chunk candidate lists.
struct ScanPlan {
  int32_t chunks;         // row chunks (grid x)
  int64_t rows_per_chunk;
  int64_t row_base;       // added to local rows in the emitted keys (index shards)
};
cudaError_t launch_scan_exact(const void* corpus, int elem, int64_t count, int dim, const void* qcodes, int nq,
                              int k, ScanPlan plan, uint64_t* cand, cudaStream_t stream);
cudaError_t launch_scan_float(const void* corpus, int elem, int64_t count, int dim, const float* queries, int nq,
                              int k, ScanPlan plan, uint64_t* cand, cudaStream_t stream);
// Merges `lists` candidate lists of k keys per query (list j of query q at
// cand + q*q_stride + j*list_stride) into the final top-k_out, best first;
// decodes (score, row) keys into the outputs (any may be null). float_keys:
// keys hold float scores; elem picks the exact-mode distance scale.
cudaError_t launch_topk_merge(const uint64_t* cand, int lists, int64_t list_stride, int64_t q_stride, int nq, int k,
                              int k_out, bool float_keys, int elem, int32_t* out_rows, int32_t* out_scores,
                              float* out_dist, uint64_t* out_keys, cudaStream_t stream);
// Exact int8 scan on the tensor cores (search_tc.cu): corpus rows and query
// codes are row_bytes apart (row_bytes >= 128, a multiple of 16, at most 1024),
// k <= 16. Writes k candidate keys per (query, part) to
// cand[(q * n_parts + part) * k], merged by launch_topk_merge with
// lists = n_parts, list_stride = k, q_stride = n_parts * k.
struct TcScanPlan {
  int32_t n_qtiles;        // 128-query tiles
  int32_t n_parts;         // contiguous corpus parts
  int64_t rows_per_part;   // a multiple of 256
};
bool scan_exact_tc_supported(int elem, int row_bytes, int k, const void* corpus, const void* qcodes);
TcScanPlan plan_scan_exact_tc(int64_t count, int nq);
// qthr (nullable): nq zeroed words the CTAs of one query share their k-th
// best scores through, so that later corpus parts skip rows early; the
// merged result does not depend on it.
cudaError_t launch_scan_exact_tc(const void* corpus, int64_t count, int row_bytes, const void* qcodes, int nq, int k,
                                 TcScanPlan plan, int64_t row_base, uint64_t* cand, uint32_t* qthr, uint32_t* err,
                                 cudaStream_t stream);

// Exact int16 scan on the tensor cores (search_tc.cu): rows and queries as
// byte planes (launch_split_int16) of plane_bytes per row (>= 128, a multiple
// of 16, at most 768); k <= 16; plan.rows_per_part a multiple of 64 (as
// plan_scan_exact_tc gives). Same candidate output as launch_scan_exact_tc.
bool scan_exact_tc16_supported(int dim, int plane_bytes, int k);
cudaError_t launch_scan_exact_tc16(const void* corpus_hi, const void* corpus_lo, int64_t count, int plane_bytes,
                                   const void* q_hi, const void* q_lo, int nq, int k, TcScanPlan plan,
                                   int64_t row_base, uint64_t* cand, uint32_t* qthr, uint32_t* err,
                                   cudaStream_t stream);
// int16 codes (rows src_row_bytes apart) -> a signed high-byte plane and an
// unsigned low-byte plane of plane_bytes per row, zero padded past dim.
cudaError_t launch_split_int16(const void* src, int64_t rows, int dim, int src_row_bytes, int plane_bytes, void* hi,
                               void* lo, cudaStream_t stream);

// Row-wise normalize (optional) + quantize (quant 1/2) or copy (quant 0) into
// rows of out_row_bytes (zero padded).
cudaError_t launch_normalize_quantize(const float* in, int64_t count, int dim, int quant, int out_row_bytes,
                                      bool normalize, void* out, cudaStream_t stream);

}  // namespace sem
