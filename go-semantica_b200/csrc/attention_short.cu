// Bidirectional attention of sequences shorter than 128 tokens on CUDA cores,
// in the reference's float32 order (MultiHeadAttentionChunked with mask nil,
// internal/kernels/attention.go:178-310, :344-363, as model_int8.go:455-500
// calls it):
//
//   score[i][j] = dotProductSIMD(q_i, k_j, 256) * scale
//     (simd_amd64.s:19-76: 8 fused lane accumulators, lane l taking elements
//     8v + l, then VEXTRACTF128 / VADDPS / VHADDPS / VHADDPS);
//   Softmax per row (activation.go:161-213): the row max, e = fastExp(s - max),
//     sum += ((e0 + e1) + e2) + e3 over groups of four and then the tail one
//     by one, p = e * (1 / sum);
//   out_i = 0; for j in order, skipping p == 0: out_i = out_i + (v_j * p)
//     (VecScaleF32 then VecAddF32: two rounded operations, no fusion).
//
// Every output is bit-identical to the reference's amd64 build. The tensor-core
// kernel (attention.cu) serves longer sequences, whose keys do not fit in
// shared memory as float32.
//
// One CTA = 8 queries of one head of one sequence. K (float32, the lanes of
// each row apart so a lane reads its 32 elements with eight 16-byte loads)
// fills shared memory for the scores; V then replaces it for the weighted sum.
// q and k are the head-normed, RoPE'd float32 rows the Q/K norm kernel writes
// back into the projection output for these rows; v is the projection output.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace sem {
namespace {

constexpr int kHd = 256;
constexpr int kAsQ = 8;            // queries per CTA
constexpr int kAsQBlocks = 16;     // 16 x 8 covers a 127-token sequence
constexpr int kAsKParts = 32 / kAsQ;  // 8-lane groups per query: each scores every kAsKParts-th key
constexpr int kAsMaxKeys = 127;    // sequences shorter than 128 tokens
constexpr int kAsThreads = 256;
constexpr int kKLane = 36;         // words per lane of a K row: 32 elements + 4 (bank spread)
constexpr int kKRow = 8 * kKLane;  // words per K row
constexpr int kAsSPWords = kAsQ * 128 + 128 * kAsQ;  // scores and probabilities
// shared memory for sequences of up to max_len keys: K rows (V rows reuse the
// space), then the scores and the probabilities
__host__ __device__ inline int as_kv_words(int max_len) { return max_len * kKRow; }
constexpr int kAsSmemMax = (kAsMaxKeys * kKRow + kAsSPWords) * 4;

__device__ __forceinline__ float group_hsum8(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

__global__ void __launch_bounds__(kAsThreads, 1)
    attention_short_kernel(const float* __restrict__ qkv, int nh, float scale, const int32_t* __restrict__ cu,
                           const int32_t* __restrict__ tile_seq, int max_len, int hw, float* __restrict__ out,
                           uint32_t* __restrict__ absmax) {
  extern __shared__ __align__(16) float as_smem[];
  float* KV = as_smem;                    // K [L][8][kKLane], then V [L][256]
  float* S = KV + as_kv_words(max_len);   // scores, then e = fastExp(s - max) [kAsQ][128]
  float* Pt = S + kAsQ * 128;         // probabilities, transposed [128][kAsQ]
  __shared__ float red[kAsThreads / 32];
  const int per_tile = nh * kAsQBlocks;
  const int tile = blockIdx.x / per_tile;
  const int h = (blockIdx.x % per_tile) / kAsQBlocks, qb = blockIdx.x % kAsQBlocks;
  const int s = tile_seq[tile];
  const int r0 = cu[s], L = cu[s + 1] - r0;
  const int q0 = qb * kAsQ;
  if (q0 >= L || L > max_len) return;  // uniform over the CTA
  const int nq = min(kAsQ, L - q0);
  const int ld = (nh + 2) * kHd;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, l = tid & 7, g = tid >> 3;

  // ---- K rows: element 8v + lane at [j][lane][v] ----
  // (loads batched eight deep: the stores wait for them, the next loads do not)
  const float* kbase = qkv + (size_t)r0 * ld + nh * kHd;
  for (int i0 = tid; i0 < L * 64; i0 += 8 * kAsThreads) {
    float4 x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kAsThreads;
      if (i < L * 64) x[u] = *reinterpret_cast<const float4*>(kbase + (size_t)(i >> 6) * ld + 4 * (i & 63));
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kAsThreads;
      if (i >= L * 64) break;
      const int j = i >> 6, p = i & 63;  // elements 4p .. 4p + 3: lanes 4 (p & 1) + e, v = p / 2
      float* dst = KV + j * kKRow + 4 * (p & 1) * kKLane + (p >> 1);
      dst[0] = x[u].x;
      dst[kKLane] = x[u].y;
      dst[2 * kKLane] = x[u].z;
      dst[3 * kKLane] = x[u].w;
    }
  }
  // ---- this group's query lane: elements 8v + l of q_i ----
  const int i = g % kAsQ, jpar = g / kAsQ;  // groups of one warp share jpar: uniform loop bounds
  float qr[32];
  if (i < nq) {
    const float* qrow = qkv + (size_t)(r0 + q0 + i) * ld + h * kHd + l;
#pragma unroll
    for (int v = 0; v < 32; ++v) qr[v] = qrow[8 * v];
  } else {
#pragma unroll
    for (int v = 0; v < 32; ++v) qr[v] = 0.0f;
  }
  __syncthreads();

  // ---- scores: four keys per pass (independent accumulation chains) ----
  for (int j0 = jpar; j0 < L; j0 += 4 * kAsKParts) {
    const float4* kr[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)  // keys past the sequence recompute its last key and are not stored
      kr[k] = reinterpret_cast<const float4*>(KV + min(j0 + kAsKParts * k, L - 1) * kKRow + l * kKLane);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 k4 = kr[k][u];
        acc[k] = __fmaf_rn(qr[4 * u], k4.x, acc[k]);
        acc[k] = __fmaf_rn(qr[4 * u + 1], k4.y, acc[k]);
        acc[k] = __fmaf_rn(qr[4 * u + 2], k4.z, acc[k]);
        acc[k] = __fmaf_rn(qr[4 * u + 3], k4.w, acc[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float d = group_hsum8(acc[k]);
      const int j = j0 + kAsKParts * k;
      if (l == 0 && i < nq && j < L) S[i * 128 + j] = __fmul_rn(d, scale);
    }
  }
  __syncthreads();  // K consumed, scores complete

  // ---- V rows (natural layout) load while the softmax runs ----
  const float* vbase = qkv + (size_t)r0 * ld + (nh + 1) * kHd;
  for (int p = tid; p < L * 64; p += kAsThreads)
    cp_async16(KV + (p >> 6) * kHd + 4 * (p & 63), vbase + (size_t)(p >> 6) * ld + 4 * (p & 63), true);
  cp_async_commit();

  // ---- softmax, one warp per row, over the row's keys [lo, hi]: every key,
  // or in a sliding-window layer those within hw positions, as one
  // contiguous row of their own (keys outside weigh nothing) ----
  for (int r = warp; r < kAsQ; r += kAsThreads / 32) {
    if (r >= nq) {  // rows past the sequence contribute nothing
      for (int j = lane; j < L; j += 32) Pt[j * kAsQ + r] = 0.0f;
      continue;
    }
    const int qpos = q0 + r;
    const int lo = max(0, qpos - hw), hi = min(L - 1, qpos + hw), n = hi - lo + 1;
    float* row = S + r * 128;
    float mx = -INFINITY;
    for (int j = lo + lane; j <= hi; j += 32) mx = fmaxf(mx, row[j]);
    mx = warp_max(mx);
    for (int j = lo + lane; j <= hi; j += 32) row[j] = fast_exp_ref(__fsub_rn(row[j], mx));
    __syncwarp();
    const int ng = n / 4;  // groups of four (at most 31: one per lane)
    float t = 0.0f;
    if (lane < ng) {
      const float* g4 = row + lo + 4 * lane;
      t = __fadd_rn(__fadd_rn(__fadd_rn(g4[0], g4[1]), g4[2]), g4[3]);
    }
    float sum = 0.0f;
    for (int k = 0; k < ng; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, t, k));
    for (int k = lo + 4 * ng; k <= hi; ++k) sum = __fadd_rn(sum, row[k]);
    const float u = sum == 0.0f ? __fdiv_rn(1.0f, (float)n) : 0.0f;
    const float inv = sum == 0.0f ? 0.0f : __fdiv_rn(1.0f, sum);
    for (int j = lane; j < L; j += 32)
      Pt[j * kAsQ + r] = (j < lo || j > hi) ? 0.0f : (sum == 0.0f ? u : __fmul_rn(row[j], inv));
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- out_i[d] for the CTA's queries, thread d ----
  const int d = tid;
  float o[kAsQ];
#pragma unroll
  for (int q = 0; q < kAsQ; ++q) o[q] = 0.0f;
  for (int j = 0; j < L; ++j) {
    const float v = KV[j * kHd + d];
    const float4* pp = reinterpret_cast<const float4*>(Pt + j * kAsQ);
#pragma unroll
    for (int q4 = 0; q4 < kAsQ / 4; ++q4) {
      const float4 p = pp[q4];
      const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float w = pv[e];
        const float a = __fadd_rn(o[4 * q4 + e], __fmul_rn(v, w));
        o[4 * q4 + e] = w == 0.0f ? o[4 * q4 + e] : a;  // the reference skips zero weights
      }
    }
  }
  float m = 0.0f;
  float* orow = out + (size_t)(r0 + q0) * (nh * kHd) + h * kHd + d;
#pragma unroll
  for (int q = 0; q < kAsQ; ++q)
    if (q < nq) {
      orow[(size_t)q * (nh * kHd)] = o[q];
      m = fmaxf(m, fabsf(o[q]));
    }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0 && absmax) {
    float mm = 0.0f;
#pragma unroll
    for (int w = 0; w < kAsThreads / 32; ++w) mm = fmaxf(mm, red[w]);
    if (mm > 0.0f) atomicMax(&absmax[s], __float_as_uint(mm));
  }
}

}  // namespace

cudaError_t launch_attention_short(const float* qkv, int num_heads, float scale, int half_window, SeqMeta meta,
                                   AttnTiles tiles, int max_len, float* out, uint32_t* absmax, cudaStream_t stream) {
  if (tiles.n_tiles == 0) return cudaSuccess;
  if (num_heads < 1 || num_heads > 3 || !qkv || !out || !meta.cu_seqlens || !tiles.tile_seq || max_len < 1 ||
      max_len > kAsMaxKeys)
    return cudaErrorInvalidValue;
  {
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
      if ((e = cudaFuncSetAttribute(attention_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kAsSmemMax)) != cudaSuccess)
        return e;
      done[dev] = true;
    }
  }
  const int64_t grid = (int64_t)tiles.n_tiles * num_heads * kAsQBlocks;
  const int smem = (as_kv_words(max_len) + kAsSPWords) * 4;
  const int hw = half_window > 0 && half_window < kAsMaxKeys ? half_window : kAsMaxKeys;
  attention_short_kernel<<<(unsigned)grid, kAsThreads, smem, stream>>>(qkv, num_heads, scale, meta.cu_seqlens,
                                                                      tiles.tile_seq, max_len, hw, out, absmax);
  return cudaGetLastError();
}

}  // namespace sem
