// Element-wise and row kernels of the EmbeddingGemma forward pass (sm_100a).
//
// Each kernel restates one step of internal/runtime/model_int8.go:148-256 so
// that its float32 results are bit-identical to the reference's Go code:
// the RMSNorm sum of squares follows the 8-lane AVX2 order, multiplies are
// unfused, divisions and square roots are IEEE-rounded (--fmad=false, no
// fast-math). Rows of a batch are packed back to back; row_seq maps a row to
// its sequence, whose activation scale is the absmax of that sequence alone
// (the reference quantises one whole sequence per call, quantize.go:29-69).
#include <cooperative_groups.h>

#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace sem {

namespace cg = cooperative_groups;

// ---------------------------------------------------------------------------
// f16 decoders. The reference has two and they differ on subnormals.
// ---------------------------------------------------------------------------

// internal/runtime/model_int8.go:571-597 (projection block scales). The
// uint16 exponent wraps while a subnormal is normalised; the shift into 32
// bits drops the wrapped bits, which gives the correctly scaled value.
__device__ __forceinline__ float f16_runtime(uint16_t f16) {
  uint16_t sign = (f16 >> 15) & 1, exponent = (f16 >> 10) & 0x1f, fraction = f16 & 0x3ff;
  if (exponent == 0) {
    if (fraction == 0) return __uint_as_float((uint32_t)sign << 31);
    while ((fraction & 0x400) == 0) {
      fraction = (uint16_t)(fraction << 1);
      exponent = (uint16_t)(exponent - 1);
    }
    exponent = (uint16_t)(exponent + 1);
    fraction &= 0x3ff;
  } else if (exponent == 0x1f) {
    return __uint_as_float(((uint32_t)sign << 31) | 0x7f800000u | ((uint32_t)fraction << 13));
  }
  uint32_t e32 = (uint32_t)exponent + (127 - 15);
  return __uint_as_float(((uint32_t)sign << 31) | (e32 << 23) | ((uint32_t)fraction << 13));
}

// internal/gguf/tensor.go:207-240 (token embedding rows through
// ParseQ8_0Block). Subnormals decode to half their value, as in the reference.
__device__ __forceinline__ float f16_gguf(uint16_t f16) {
  uint32_t sign = (f16 >> 15) & 1, exp = (f16 >> 10) & 0x1f, mant = f16 & 0x3ff, bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign << 31;
    } else {
      uint32_t e = 127 - 15, m = mant;
      while ((m & 0x400) == 0) {
        m <<= 1;
        e--;
      }
      bits = (sign << 31) | (e << 23) | ((m & 0x3ff) << 13);
    }
  } else if (exp == 0x1f) {
    bits = (sign << 31) | (0xffu << 23) | (mant << 13);
  } else {
    bits = (sign << 31) | (((exp - 15 + 127) & 0xff) << 23) | (mant << 13);
  }
  return __uint_as_float(bits);
}

// ---------------------------------------------------------------------------
// Q8_0 repack: one thread per 34-byte block.
// ---------------------------------------------------------------------------
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ raw, int64_t rows, int nb, int8_t* __restrict__ codes,
                                   float* __restrict__ scales, int64_t dst_row_offset, int interleave, int part,
                                   bool gguf_decoder) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nb) return;
  int64_t r = i / nb;
  int b = (int)(i % nb);
  const uint8_t* blk = raw + i * 34;
  const uint16_t* p16 = reinterpret_cast<const uint16_t*>(blk);  // 34-byte blocks are 2-byte aligned
  uint16_t h = p16[0];
  int64_t dr = interleave > 0 ? (r / interleave) * (2 * interleave) + part * interleave + (r % interleave) : r;
  dr += dst_row_offset;
  scales[dr * nb + b] = gguf_decoder ? f16_gguf(h) : f16_runtime(h);
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) w[k] = (uint32_t)p16[1 + 2 * k] | ((uint32_t)p16[2 + 2 * k] << 16);
  uint4* dst = reinterpret_cast<uint4*>(codes + dr * (int64_t)nb * 32 + (int64_t)b * 32);
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

cudaError_t launch_repack_q8_0(const uint8_t* raw, int64_t rows, int cols, int8_t* dst_codes, float* dst_scales,
                               int64_t dst_row_offset, int interleave, int part, bool gguf_decoder,
                               cudaStream_t stream) {
  int nb = cols / 32;
  int64_t n = rows * nb;
  int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  repack_q8_0_kernel<<<(unsigned)blocks, threads, 0, stream>>>(raw, rows, nb, dst_codes, dst_scales,
                                                                 dst_row_offset, interleave, part, gguf_decoder);
  return cudaGetLastError();
}

// Projection weights: fp16 codes and fp32 block scales, one thread per block.
__global__ void repack_q8_0_f16_kernel(const uint8_t* __restrict__ raw, int64_t rows, int nb, __half* __restrict__ codes,
                                       float* __restrict__ scales, int64_t dst_row_offset) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nb) return;
  int64_t r = i / nb;
  int b = (int)(i % nb);
  const uint8_t* blk = raw + i * 34;
  const uint16_t h = reinterpret_cast<const uint16_t*>(blk)[0];  // 34-byte blocks are 2-byte aligned
  const int64_t dr = dst_row_offset + r;
  scales[dr * nb + b] = f16_runtime(h);
  __align__(16) __half v[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = __int2half_rn((int)(int8_t)blk[2 + k]);
  uint4* dst = reinterpret_cast<uint4*>(codes + dr * (int64_t)nb * 32 + (int64_t)b * 32);
  const uint4* src = reinterpret_cast<const uint4*>(v);
#pragma unroll
  for (int k = 0; k < 4; ++k) dst[k] = src[k];
}

cudaError_t launch_repack_q8_0_f16(const uint8_t* raw, int64_t rows, int cols, __half* dst_codes, float* dst_scales,
                                   int64_t dst_row_offset, cudaStream_t stream) {
  int nb = cols / 32;
  int64_t n = rows * nb;
  int64_t blocks = (n + 255) / 256;
  repack_q8_0_f16_kernel<<<(unsigned)blocks, 256, 0, stream>>>(raw, rows, nb, dst_codes, dst_scales, dst_row_offset);
  return cudaGetLastError();
}

// Projection weights for the split-plane GEMM (gemm_split.cu): one warp per
// row. w = q * d (exact in float32: an int8 times an fp16) is scaled by the
// power of two 2^S that puts the row's largest |w| in [2^13, 2^14); then
// hi = fp16(w * 2^S), lo = fp16(w * 2^S - hi) (the difference is exact) and
// row_scale = 2^-S.
__global__ void repack_q8_0_split_kernel(const uint8_t* __restrict__ raw, int64_t rows, int nb,
                                         __half* __restrict__ hi, __half* __restrict__ lo,
                                         float* __restrict__ row_scale, int64_t dst_row_offset) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;  // whole warps: rows is warp-uniform
  const uint8_t* row = raw + r * nb * 34;
  float m = 0.0f;
  for (int b = lane; b < nb; b += 32) {
    const uint8_t* blk = row + (int64_t)b * 34;
    const float d = fabsf(f16_runtime((uint16_t)(blk[0] | (blk[1] << 8))));
    int qm = 0;
    for (int k = 0; k < 32; ++k) qm = max(qm, abs((int)(int8_t)blk[2 + k]));
    m = fmaxf(m, __fmul_rn((float)qm, d));
  }
  m = warp_max(m);
  int e = 0;
  if (m > 0.0f) frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
  const int S = m > 0.0f ? 14 - e : 0;
  const int64_t dr = dst_row_offset + r;
  if (lane == 0) row_scale[dr] = ldexpf(1.0f, -S);
  for (int b = lane; b < nb; b += 32) {
    const uint8_t* blk = row + (int64_t)b * 34;
    const float d = f16_runtime((uint16_t)(blk[0] | (blk[1] << 8)));
    __align__(16) __half vh[32], vl[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float w = ldexpf(__fmul_rn((float)(int8_t)blk[2 + k], d), S);
      const __half h = __float2half_rn(w);
      vh[k] = h;
      vl[k] = __float2half_rn(__fsub_rn(w, __half2float(h)));
    }
    uint4* dh = reinterpret_cast<uint4*>(hi + dr * (int64_t)nb * 32 + (int64_t)b * 32);
    uint4* dl = reinterpret_cast<uint4*>(lo + dr * (int64_t)nb * 32 + (int64_t)b * 32);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      dh[k] = reinterpret_cast<const uint4*>(vh)[k];
      dl[k] = reinterpret_cast<const uint4*>(vl)[k];
    }
  }
}

cudaError_t launch_repack_q8_0_split(const uint8_t* raw, int64_t rows, int cols, __half* hi, __half* lo,
                                     float* row_scale, int64_t dst_row_offset, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const int nb = cols / 32;
  const int64_t threads = rows * 32;
  repack_q8_0_split_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(raw, rows, nb, hi, lo, row_scale,
                                                                                   dst_row_offset);
  return cudaGetLastError();
}

__global__ void gather_i32_kernel(const int32_t* __restrict__ src, const int32_t* __restrict__ idx,
                                  int32_t* __restrict__ dst, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[idx[i]];
}

cudaError_t launch_gather_i32(const int32_t* src, const int32_t* idx, int32_t* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  gather_i32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(src, idx, dst, n);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Token embedding: DequantizeQ8_0Row then the sqrt(H) scale
// (model_int8.go:167-184, gguf/tensor.go:157-177). 16 elements per thread.
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int32_t* __restrict__ ids, const int8_t* __restrict__ emb_codes,
                             const float* __restrict__ emb_scales, int vocab, int H, float* __restrict__ hidden,
                             int T, float sf, uint32_t* err_flag) {
  int per_row = H / 16;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * per_row) return;
  int row = (int)(i / per_row), c = (int)(i % per_row) * 16;
  int id = ids[row];
  float4* out = reinterpret_cast<float4*>(hidden + (int64_t)row * H + c);
  if (id < 0 || id >= vocab) {  // rejected on the host first; never read out of bounds
    if (err_flag) atomicOr(err_flag, 1u);
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    out[0] = z; out[1] = z; out[2] = z; out[3] = z;
    return;
  }
  int4 q = *reinterpret_cast<const int4*>(emb_codes + (int64_t)id * H + c);
  float s = emb_scales[(int64_t)id * (H / 32) + c / 32];
  const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
  float v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = __fmul_rn(__fmul_rn((float)qb[k], s), sf);
  out[0] = make_float4(v[0], v[1], v[2], v[3]);
  out[1] = make_float4(v[4], v[5], v[6], v[7]);
  out[2] = make_float4(v[8], v[9], v[10], v[11]);
  out[3] = make_float4(v[12], v[13], v[14], v[15]);
}

cudaError_t launch_embed(const int32_t* ids, const int8_t* emb_codes, const float* emb_scales, int vocab, int H,
                         float* hidden, int T, uint32_t* err_flag, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  int64_t n = (int64_t)T * (H / 16);
  int threads = 256;
  float sf = (float)sqrt((double)H);  // float32(math.Sqrt(float64(embDim)))
  embed_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(ids, emb_codes, emb_scales, vocab,
                                                                                 H, hidden, T, sf, err_flag);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Row statistics: 8 lanes per row, 4 rows per warp.
// ---------------------------------------------------------------------------
// Horizontal sum of the 8 lane accumulators of a row group in the order of
// dotProductAVX2Asm's VEXTRACTF128/VADDPS/VHADDPS tail (simd_amd64.s:19-76).
__device__ __forceinline__ float group_sum8_avx_order(float acc) {
  const unsigned full = 0xffffffffu;
  float hi = __shfl_down_sync(full, acc, 4, 8);
  float s = __fadd_rn(acc, hi);
  float s1 = __shfl_down_sync(full, s, 1, 8);
  float p = __fadd_rn(s, s1);
  float p2 = __shfl_down_sync(full, p, 2, 8);
  return __shfl_sync(full, __fadd_rn(p, p2), 0, 8);
}

__device__ __forceinline__ float group_max8(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4, 8));
  return v;
}

// The 4 row groups of a warp fold their row maxima into the per-sequence
// absmax: one atomic per warp when all four rows share a sequence, one per row
// otherwise. row < 0 marks an idle group. Called by all 32 lanes.
__device__ __forceinline__ void warp_seq_atomic_max(uint32_t* absmax, const int32_t* row_seq, int64_t row, float m) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  int seq = row >= 0 ? row_seq[row] : -1;
  int s0 = __shfl_sync(full, seq, 0);
  if (__all_sync(full, seq == s0)) {
    m = warp_max(m);
    if (lane == 0 && s0 >= 0) atomicMax(&absmax[s0], __float_as_uint(m));
  } else if ((lane & 7) == 0 && seq >= 0) {
    atomicMax(&absmax[seq], __float_as_uint(m));
  }
}

__global__ void row_stats_kernel(const float* __restrict__ x, const float* __restrict__ w, int H, float eps,
                                 SeqMeta meta, float* __restrict__ inv_rms, uint32_t* __restrict__ absmax) {
  int lane = threadIdx.x & 31, sub = lane & 7;
  int64_t group = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  int64_t ngroups = ((int64_t)gridDim.x * blockDim.x) >> 3;
  int64_t rounds = ((int64_t)meta.T + ngroups - 1) / ngroups;
  for (int64_t it = 0; it < rounds; ++it) {  // every lane runs every round: shuffles stay converged
    int64_t row = group + it * ngroups;
    bool valid = row < meta.T;
    const float* xr = x + (valid ? row : 0) * (int64_t)H;
    float ss = row_sumsq_ref(xr, H, sub);
    float inv = rms_inv_ref(ss, H, eps);
    float m = 0.0f;
    if (absmax) {
      for (int v = 0; v < H / 8; ++v) {
        int e = 8 * v + sub;
        m = fmaxf(m, fabsf(__fmul_rn(__fmul_rn(xr[e], inv), w[e])));
      }
      m = group_max8(m);
    }
    if (valid && sub == 0) inv_rms[row] = inv;
    if (absmax) warp_seq_atomic_max(absmax, meta.row_seq, valid ? row : -1, m);
  }
}

static unsigned row_grid(int64_t T) {
  int64_t groups = T;  // one 8-lane group per row
  int64_t blocks = (groups * 8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

cudaError_t launch_row_stats(const float* x, const float* w, int H, float eps, SeqMeta meta, float* inv_rms,
                             uint32_t* absmax, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  row_stats_kernel<<<row_grid(meta.T), 256, 0, stream>>>(x, w, H, eps, meta, inv_rms, absmax);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Quantisation with the per-sequence scale; 16 elements per thread.
// ---------------------------------------------------------------------------
// One warp per row: the sequence's scale is computed once, the row moves as
// 16-byte loads (x, and the norm weight) and 8-byte stores of four fp16 codes.
constexpr int kQuantWarps = 8;
constexpr int kQuantBatch = 9;  // float4 loads in flight per lane (a 1152-wide row in one batch)

__global__ void __launch_bounds__(kQuantWarps * 32)
    quantize_kernel(const float* __restrict__ x, const float* __restrict__ inv_rms, const float* __restrict__ w,
                    int K, SeqMeta meta, const uint32_t* __restrict__ absmax, __half* __restrict__ codes) {
  const int lane = threadIdx.x & 31;
  const int q4 = K / 4;
  const int64_t nwarps = (int64_t)gridDim.x * kQuantWarps;
  for (int64_t row = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5); row < meta.T; row += nwarps) {
    float scale, inv;
    seq_scale_ref(absmax[meta.row_seq ? meta.row_seq[row] : 0], &scale, &inv);
    const float r = inv_rms ? inv_rms[row] : 0.0f;
    const float4* xr = reinterpret_cast<const float4*>(x + row * K);
    for (int seg = 0; seg < q4; seg += 32 * kQuantBatch) {
    float4 v[kQuantBatch];
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int c4 = seg + b * 32 + lane;
      v[b] = c4 < q4 ? xr[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int b = 0; b < kQuantBatch; ++b) {
      const int c4 = seg + b * 32 + lane;
      if (c4 >= q4) continue;
      float4 e = v[b];
      if (inv_rms) {
        const float4 wv = reinterpret_cast<const float4*>(w)[c4];
        e = make_float4(__fmul_rn(__fmul_rn(e.x, r), wv.x), __fmul_rn(__fmul_rn(e.y, r), wv.y),
                        __fmul_rn(__fmul_rn(e.z, r), wv.z), __fmul_rn(__fmul_rn(e.w, r), wv.w));
      }
      *reinterpret_cast<uint2*>(codes + row * K + 4 * c4) = quant_codes4(e, inv);
    }
    }
  }
}

// Blocks of one full wave of a grid-stride kernel on the current device (its
// resident blocks per SM x the SMs), cached per device: a larger grid leaves
// a partial last wave running alone.
template <class Kern>
static int64_t wave_blocks(Kern kernel, int threads, std::atomic<int>* cache) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    int per_sm = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    n = per_sm * sms;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

cudaError_t launch_quantize(const float* x, const float* inv_rms, const float* w, int K, SeqMeta meta,
                            const uint32_t* absmax, __half* codes, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  if (K % 4 != 0) return cudaErrorInvalidValue;
  static std::atomic<int> wave[64];
  int64_t blocks = (meta.T + kQuantWarps - 1) / kQuantWarps;
  const int64_t full = wave_blocks(quantize_kernel, kQuantWarps * 32, wave);
  if (blocks > full) blocks = full;
  quantize_kernel<<<(unsigned)blocks, kQuantWarps * 32, 0, stream>>>(x, inv_rms, w, K, meta, absmax, codes);
  return cudaGetLastError();
}

// absMaxScalar over a whole buffer (quantize.go:80-90) into slot[0].
__global__ void absmax_kernel(const float* __restrict__ x, int64_t n, uint32_t* __restrict__ slot) {
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(slot, __float_as_uint(m));
}

cudaError_t launch_absmax(const float* x, int64_t n, uint32_t* slot, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  absmax_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, n, slot);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Q/K head norms + RoPE + fp16 split (model_int8.go:371-452, rope_cache.go).
// One warp per row: lane group g (8 lanes) owns q head g (g < nh) or the k head
// (g == nh). Lane `sub` holds elements 8v+sub, so RoPE partners i and i+128
// (v and v+16) sit in the same lane.
// ---------------------------------------------------------------------------
constexpr int kHeadDim = 256;

constexpr int kHeadPad = kHeadDim + 8;  // head stride in shared memory: 4 heads on distinct banks
constexpr int kQkWarps = 8;

__global__ void __launch_bounds__(kQkWarps * 32)
    qk_norm_rope_kernel(float* __restrict__ qkv, const float* __restrict__ q_norm,
                        const float* __restrict__ k_norm, const float* __restrict__ rope_cos,
                        const float* __restrict__ rope_sin, float eps, int nh, SeqMeta meta,
                        __half* __restrict__ qh, __half* __restrict__ ql, __half* __restrict__ kh,
                        __half* __restrict__ kl, __half* __restrict__ vh, __half* __restrict__ vl,
                        int64_t f32_row0, int64_t v_row0) {
  __shared__ __align__(16) float sh[kQkWarps][4 * kHeadPad];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 3, sub = lane & 7;
  const int64_t nwarps = (int64_t)gridDim.x * kQkWarps;
  const int ld = (nh + 2) * kHeadDim;
  float* rowbuf = sh[warp];
  const bool active = g <= nh;
  const float* wn = g < nh ? q_norm : k_norm;
  for (int64_t row = (int64_t)blockIdx.x * kQkWarps + warp; row < meta.T; row += nwarps) {  // uniform per warp
    float* base = qkv + row * ld;
    // q heads and the k head into shared memory (64 float4 per head)
    for (int idx = lane; idx < (nh + 1) * 64; idx += 32) {
      const int hd = idx >> 6, c4 = idx & 63;
      *reinterpret_cast<float4*>(rowbuf + hd * kHeadPad + 4 * c4) = reinterpret_cast<const float4*>(base)[idx];
    }
    __syncwarp();
    const float* x = rowbuf + (active ? g : nh) * kHeadPad;
    float acc = 0.0f;
#pragma unroll 8
    for (int v = 0; v < kHeadDim / 8; ++v) {
      const float t = x[8 * v + sub];
      acc = fmaf(t, t, acc);
    }
    const float inv = rms_inv_ref(group_sum8_avx_order(acc), kHeadDim, eps);
    if (active) {
      const int pos = meta.row_pos[row];
      const float4* cs = reinterpret_cast<const float4*>(rope_cos + (int64_t)pos * (kHeadDim / 2));
      const float4* sn = reinterpret_cast<const float4*>(rope_sin + (int64_t)pos * (kHeadDim / 2));
      __half* dh = g < nh ? qh + (row * nh + g) * kHeadDim : kh + row * kHeadDim;
      __half* dl = g < nh ? ql + (row * nh + g) * kHeadDim : kl + row * kHeadDim;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = 4 * sub + 32 * k;  // NeoX pairs (i, i + 128)
        float a0[4], a1[4];
        *reinterpret_cast<float4*>(a0) = *reinterpret_cast<const float4*>(x + i);
        *reinterpret_cast<float4*>(a1) = *reinterpret_cast<const float4*>(x + i + 128);
        float c[4], s[4];
        *reinterpret_cast<float4*>(c) = cs[i / 4];
        *reinterpret_cast<float4*>(s) = sn[i / 4];
        float w0[4] = {1.f, 1.f, 1.f, 1.f}, w1[4] = {1.f, 1.f, 1.f, 1.f};
        if (wn) {
          *reinterpret_cast<float4*>(w0) = reinterpret_cast<const float4*>(wn + i)[0];
          *reinterpret_cast<float4*>(w1) = reinterpret_cast<const float4*>(wn + i + 128)[0];
        }
        __half2 h0[2], l0[2], h1[2], l1[2];
        float f0[4], f1[4];  // the float32 results, kept for rows of short sequences
#pragma unroll
        for (int u = 0; u < 4; u += 2) {
          float r0[2], r1[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            // the reference skips a head norm whose weight tensor is absent (model_int8.go:374, :408)
            const float x0 = wn ? __fmul_rn(__fmul_rn(a0[u + z], inv), w0[u + z]) : a0[u + z];
            const float x1 = wn ? __fmul_rn(__fmul_rn(a1[u + z], inv), w1[u + z]) : a1[u + z];
            r0[z] = __fsub_rn(__fmul_rn(x0, c[u + z]), __fmul_rn(x1, s[u + z]));
            r1[z] = __fadd_rn(__fmul_rn(x0, s[u + z]), __fmul_rn(x1, c[u + z]));
            f0[u + z] = r0[z];
            f1[u + z] = r1[z];
          }
          __half a, b, e2, f;
          split_half(r0[0], a, b);
          split_half(r0[1], e2, f);
          h0[u / 2] = __halves2half2(a, e2);
          l0[u / 2] = __halves2half2(b, f);
          split_half(r1[0], a, b);
          split_half(r1[1], e2, f);
          h1[u / 2] = __halves2half2(a, e2);
          l1[u / 2] = __halves2half2(b, f);
        }
        *reinterpret_cast<uint2*>(dh + i) = *reinterpret_cast<uint2*>(h0);
        *reinterpret_cast<uint2*>(dl + i) = *reinterpret_cast<uint2*>(l0);
        *reinterpret_cast<uint2*>(dh + i + 128) = *reinterpret_cast<uint2*>(h1);
        *reinterpret_cast<uint2*>(dl + i + 128) = *reinterpret_cast<uint2*>(l1);
        if (row >= f32_row0) {  // the float32 attention of short sequences reads these back in place
          float* dst = base + g * kHeadDim;  // q head g, or the k head right after the q heads
          *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(f0);
          *reinterpret_cast<float4*>(dst + i + 128) = *reinterpret_cast<const float4*>(f1);
        }
      }
    }
    // v: all 32 lanes, 8 consecutive elements each (rows below v_row0: the
    // projection wrote the planes)
    if (row >= v_row0) {
      const float4* vx = reinterpret_cast<const float4*>(base + (nh + 1) * kHeadDim + lane * 8);
      float vv[8];
      *reinterpret_cast<float4*>(vv) = vx[0];
      *reinterpret_cast<float4*>(vv + 4) = vx[1];
      __half hv[8], lv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) split_half(vv[k], hv[k], lv[k]);
      *reinterpret_cast<uint4*>(vh + row * kHeadDim + lane * 8) = *reinterpret_cast<uint4*>(hv);
      *reinterpret_cast<uint4*>(vl + row * kHeadDim + lane * 8) = *reinterpret_cast<uint4*>(lv);
    }
    __syncwarp();  // the row buffer is reloaded next
  }
}

cudaError_t launch_qk_norm_rope(float* qkv, const float* q_norm, const float* k_norm, const float* rope_cos,
                                const float* rope_sin, float eps, int num_heads, SeqMeta meta, __half* qh,
                                __half* ql, __half* kh, __half* kl, __half* vh, __half* vl, int64_t f32_row0,
                                int64_t v_row0, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  if (num_heads < 1 || num_heads > 3) return cudaErrorInvalidValue;
  int64_t blocks = (meta.T + kQkWarps - 1) / kQkWarps;
  if (blocks > 148 * 8) blocks = 148 * 8;
  qk_norm_rope_kernel<<<(unsigned)blocks, kQkWarps * 32, 0, stream>>>(qkv, q_norm, k_norm, rope_cos, rope_sin, eps, num_heads,
                                                            meta, qh, ql, kh, kl, vh, vl, f32_row0, v_row0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Post-norm + residual (model_int8.go:202-210, :224-232) fused with the next
// RMSNorm (:194 / :216 of the following step) and its INT8 quantisation
// (QuantizeSymmetricINT8Into, quantize.go:29-69: one scale per sequence).
// ---------------------------------------------------------------------------
// A cluster of kRqCluster CTAs owns one sequence at a time, each CTA a
// contiguous share of its rows; as many clusters as fit loop over the
// sequences.
//  Phase 1, one warp per pair of rows: hidden = rmsnorm(o, post_w) + hidden,
//   the next norm's inv_rms, and the CTA's max |(hidden * inv_rms) * next_w|.
//  The CTA maxima meet in rank 0's shared memory (distributed shared memory
//   atomics); after one cluster barrier every CTA holds the sequence absmax.
//  Phase 2 re-reads the CTA's rows of hidden (just written: L2 hits) and
//   writes the INT8 codes (as fp16, the projection operand type).
// Without codes the kernel ends after phase 1 (the last layer, whose rows go
// to output_norm and the pool).
//
// The sums of squares keep the reference's 8-lane AVX2 order: lane `sub` of a
// row's 8-lane group accumulates elements 8v + sub for v = 0, 1, ... with fused
// multiply-adds, then the lanes combine in dotProductAVX2Asm's tail order
// (norm.go:8-36, simd_amd64.s:19-76). The rows sit in shared memory
// transposed to [residue][v], so a lane reads its chain 16 bytes at a time.
constexpr int kRqWarps = 8;
constexpr int kRqCluster = 8;

template <int H>
struct RqShape {
  static constexpr int kNV = H / 128;                   // float4 per lane per row
  static constexpr int kTS = H / 8 + 4;                 // floats per residue column: conflict-free
  static constexpr int kWarpFloats = 2 * 8 * kTS;       // two rows per warp
  static constexpr int kSmem = kRqWarps * kWarpFloats * 4;
};

// Sum of squares of one residue column in element order (one lane's chain).
template <int H>
__device__ __forceinline__ float chain_sumsq(const float* col) {
  float acc = 0.0f;
#pragma unroll 2
  for (int j = 0; j < H / 32; ++j) {
    const float4 t = *reinterpret_cast<const float4*>(col + 4 * j);
    acc = fmaf(t.x, t.x, acc);
    acc = fmaf(t.y, t.y, acc);
    acc = fmaf(t.z, t.z, acc);
    acc = fmaf(t.w, t.w, acc);
  }
  return acc;
}

template <int H>
__global__ void __cluster_dims__(kRqCluster, 1, 1) __launch_bounds__(kRqWarps * 32, 2)
    residual_quant_kernel(const float* __restrict__ o, const float* __restrict__ post_w, float* hidden,
                          const float* __restrict__ next_w, float eps, SeqMeta meta, float* inv_rms,
                          uint32_t* __restrict__ absmax, __half* __restrict__ codes) {
  using S = RqShape<H>;
  constexpr int NV = S::kNV, TS = S::kTS;
  extern __shared__ float4 rq_smem[];
  __shared__ uint32_t s_warpmax[kRqWarps];
  __shared__ uint32_t s_seqmax[3];  // rank 0's slots, rotated per sequence
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 3, sub = lane & 7;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  float* rows = reinterpret_cast<float*>(rq_smem) + warp * S::kWarpFloats;
  const float* chain = rows + (g & 1) * 8 * TS + sub * TS;  // groups 2, 3 repeat rows 0, 1
  const bool quant = codes != nullptr;
  if (quant) {
    if (crank == 0 && threadIdx.x < 3) s_seqmax[threadIdx.x] = 0u;
    cluster.sync();
  }
  const int nclusters = gridDim.x / kRqCluster;
  int it = 0;
  for (int s = blockIdx.x / kRqCluster; s < meta.B; s += nclusters, ++it) {  // uniform over the cluster
    const int a = meta.cu_seqlens[s], len = meta.cu_seqlens[s + 1] - a;
    const int share = (len + kRqCluster - 1) / kRqCluster;
    const int r0 = a + min(len, crank * share), r1 = a + min(len, (crank + 1) * share);
    float tmax = 0.0f;
    for (int row0 = r0 + 2 * warp; row0 < r1; row0 += 2 * kRqWarps) {  // uniform per warp
      const bool has1 = row0 + 1 < r1;
      // lane's float4 b of the pair: row b / NV, column 4 * lane + 128 * (b % NV)
      const int64_t lane_off = (int64_t)row0 * H + 4 * lane;
      float* lane_col = rows + 4 * (lane & 1) * TS + (lane >> 1);
      // o rows into shared memory (transposed)
#pragma unroll
      for (int b = 0; b < 2 * NV; ++b) {
        const int rr = b / NV, cb = b % NV;
        const float4 ov = rr == 0 || has1 ? *reinterpret_cast<const float4*>(o + lane_off + rr * H + 128 * cb)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        // element 4*c4 + k (c4 = 32 cb + lane) has residue 4*(lane & 1) + k and index v = 16 cb + lane / 2
        float* col = lane_col + rr * 8 * TS + 16 * cb;
        col[0] = ov.x;
        col[TS] = ov.y;
        col[2 * TS] = ov.z;
        col[3 * TS] = ov.w;
      }
      // The hidden rows load while the first chains run. The compiler barrier
      // keeps these loads after the o stores: o and hidden in registers at once
      // would halve the CTAs per SM.
      asm volatile("" ::: "memory");
      float4 hv[2 * NV];
#pragma unroll
      for (int b = 0; b < 2 * NV; ++b) {
        const int rr = b / NV, cb = b % NV;
        hv[b] = rr == 0 || has1 ? *reinterpret_cast<const float4*>(hidden + lane_off + rr * H + 128 * cb)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncwarp();
      const float inv1 = rms_inv_ref(group_sum8_avx_order(chain_sumsq<H>(chain)), H, eps);
      const float i1[2] = {__shfl_sync(full, inv1, 0), __shfl_sync(full, inv1, 8)};
      __syncwarp();  // every chain has read o before the new rows replace it
#pragma unroll
      for (int b = 0; b < 2 * NV; ++b) {
        const int rr = b / NV, cb = b % NV;
        float* col = lane_col + rr * 8 * TS + 16 * cb;
        float4 ov = make_float4(col[0], col[TS], col[2 * TS], col[3 * TS]);
        if (post_w) {  // an absent post-norm leaves o as it is (model_int8.go:203, :225)
          const float4 w = *reinterpret_cast<const float4*>(post_w + 4 * lane + 128 * cb);
          ov = make_float4(__fmul_rn(__fmul_rn(ov.x, i1[rr]), w.x), __fmul_rn(__fmul_rn(ov.y, i1[rr]), w.y),
                           __fmul_rn(__fmul_rn(ov.z, i1[rr]), w.z), __fmul_rn(__fmul_rn(ov.w, i1[rr]), w.w));
        }
        const float4 h = hv[b];
        const float4 nh = make_float4(__fadd_rn(ov.x, h.x), __fadd_rn(ov.y, h.y), __fadd_rn(ov.z, h.z),
                                      __fadd_rn(ov.w, h.w));
        if (rr == 0 || has1) *reinterpret_cast<float4*>(hidden + lane_off + rr * H + 128 * cb) = nh;
        hv[b] = nh;
        col[0] = nh.x;
        col[TS] = nh.y;
        col[2 * TS] = nh.z;
        col[3 * TS] = nh.w;
      }
      __syncwarp();
      const float inv2 = rms_inv_ref(group_sum8_avx_order(chain_sumsq<H>(chain)), H, eps);
      if (sub == 0 && (g == 0 || (g == 1 && has1))) inv_rms[row0 + g] = inv2;
      if (quant) {  // rows past the share are zeros: |0 * inv * w| = 0
        const float i2[2] = {__shfl_sync(full, inv2, 0), __shfl_sync(full, inv2, 8)};
#pragma unroll
        for (int b = 0; b < 2 * NV; ++b) {
          const int rr = b / NV, cb = b % NV;
          const float4 w = *reinterpret_cast<const float4*>(next_w + 4 * lane + 128 * cb);
          const float4 h = hv[b];
          tmax = fmaxf(tmax, fabsf(__fmul_rn(__fmul_rn(h.x, i2[rr]), w.x)));
          tmax = fmaxf(tmax, fabsf(__fmul_rn(__fmul_rn(h.y, i2[rr]), w.y)));
          tmax = fmaxf(tmax, fabsf(__fmul_rn(__fmul_rn(h.z, i2[rr]), w.z)));
          tmax = fmaxf(tmax, fabsf(__fmul_rn(__fmul_rn(h.w, i2[rr]), w.w)));
        }
      }
      __syncwarp();  // the chains are done before the next pair is stored
    }
    if (!quant) continue;
    // sequence absmax: warp, CTA, then cluster (rank 0's slot it % 3)
    tmax = warp_max(tmax);
    if (lane == 0) s_warpmax[warp] = __float_as_uint(tmax);
    // Slot (it + 1) % 3 was last read before the barrier of the previous
    // sequence, which rank 0 has passed; zero it for the next sequence.
    if (crank == 0 && threadIdx.x == 0) s_seqmax[(it + 1) % 3] = 0u;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t m = 0;
#pragma unroll
      for (int w = 0; w < kRqWarps; ++w) m = max(m, s_warpmax[w]);
      atomicMax(cluster.map_shared_rank(&s_seqmax[it % 3], 0), m);
    }
    cluster.sync();  // release/acquire: the maxima, hidden and inv_rms of every CTA
    const uint32_t mbits = *cluster.map_shared_rank(&s_seqmax[it % 3], 0);
    if (crank == 0 && threadIdx.x == 0) absmax[s] = mbits;
    float scale, qinv;
    seq_scale_ref(mbits, &scale, &qinv);
    // phase 2: codes = quantize((hidden * inv_rms) * next_w), a warp per row
    for (int row = r0 + warp; row < r1; row += kRqWarps) {  // uniform per warp
      const float r = inv_rms[row];
      const int64_t lane_off = (int64_t)row * H + 4 * lane;
      float4 v[NV];
#pragma unroll
      for (int b = 0; b < NV; ++b) v[b] = *reinterpret_cast<const float4*>(hidden + lane_off + 128 * b);
#pragma unroll
      for (int b = 0; b < NV; ++b) {
        const float4 w = *reinterpret_cast<const float4*>(next_w + 4 * lane + 128 * b);
        const float4 x = make_float4(__fmul_rn(__fmul_rn(v[b].x, r), w.x), __fmul_rn(__fmul_rn(v[b].y, r), w.y),
                                     __fmul_rn(__fmul_rn(v[b].z, r), w.z), __fmul_rn(__fmul_rn(v[b].w, r), w.w));
        *reinterpret_cast<uint2*>(codes + lane_off + 128 * b) = quant_codes4(x, qinv);
      }
    }
  }
  if (quant) cluster.sync();  // rank 0's slots stay alive until every CTA has read them
}

template <int H>
static cudaError_t launch_rq(const float* o, const float* post_w, float* hidden, const float* next_w, float eps,
                             SeqMeta meta, float* inv_rms, uint32_t* absmax, __half* codes, cudaStream_t stream) {
  auto fn = residual_quant_kernel<H>;
  const int smem = RqShape<H>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  // as many clusters as fit at once, each looping over sequences (measured
  // ~3 % faster than one cluster per sequence); cached per device
  static int resident_of[64];
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int resident = __atomic_load_n(&resident_of[dev], __ATOMIC_RELAXED);
  if (resident == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kRqCluster * 148, 1, 1);
    cfg.blockDim = dim3(kRqWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    if ((e = cudaOccupancyMaxActiveClusters(&resident, fn, &cfg)) != cudaSuccess) return e;
    if (resident < 1) return cudaErrorInvalidConfiguration;
    __atomic_store_n(&resident_of[dev], resident, __ATOMIC_RELAXED);
  }
  const int clusters = meta.B < resident ? meta.B : resident;
  fn<<<(unsigned)(clusters * kRqCluster), kRqWarps * 32, smem, stream>>>(o, post_w, hidden, next_w, eps, meta,
                                                                          inv_rms, absmax, codes);
  return cudaGetLastError();
}

cudaError_t launch_residual_norm(const float* o, const float* post_w, float* hidden, const float* next_w, int H,
                                 float eps, SeqMeta meta, float* inv_rms, uint32_t* absmax, __half* codes,
                                 cudaStream_t stream) {
  if (meta.T == 0 || meta.B == 0) return cudaSuccess;
  if ((absmax == nullptr) != (codes == nullptr) || (codes && !next_w) || !meta.cu_seqlens) return cudaErrorInvalidValue;
  switch (H) {
    case 256: return launch_rq<256>(o, post_w, hidden, next_w, eps, meta, inv_rms, absmax, codes, stream);
    case 512: return launch_rq<512>(o, post_w, hidden, next_w, eps, meta, inv_rms, absmax, codes, stream);
    case 768: return launch_rq<768>(o, post_w, hidden, next_w, eps, meta, inv_rms, absmax, codes, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// output_norm + MeanPoolingPartial + l2Normalize (model_int8.go:235-255,
// attention.go:423-445, model.go:808-820). One block per sequence; each
// thread sums its columns over the rows in order, one thread does the
// sequential sum of squares.
// ---------------------------------------------------------------------------
__global__ void pool_l2_kernel(const float* __restrict__ hidden, const float* __restrict__ inv_rms,
                               const float* __restrict__ w, int H, SeqMeta meta, const int32_t* __restrict__ out_dims,
                               const int64_t* __restrict__ out_offsets, float* __restrict__ out) {
  extern __shared__ float pooled[];
  __shared__ float s_norm;
  int s = blockIdx.x;
  int r0 = meta.cu_seqlens[s], r1 = meta.cu_seqlens[s + 1];
  const bool l2 = out_dims != nullptr;  // else: every column, no normalisation (the dense head's input)
  int od = l2 ? out_dims[s] : H;
  float scale = __fdiv_rn(1.0f, (float)(r1 - r0));
  for (int i = threadIdx.x; i < od; i += blockDim.x) {
    float acc = 0.0f;
    float wi = w ? w[i] : 1.0f;
    for (int r = r0; r < r1; ++r) {
      float x = hidden[(int64_t)r * H + i];
      float nv = w ? __fmul_rn(__fmul_rn(x, inv_rms[r]), wi) : x;
      acc = __fadd_rn(acc, nv);
    }
    pooled[i] = __fmul_rn(acc, scale);
  }
  __syncthreads();
  if (!l2) {
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(int64_t)s * H + i] = pooled[i];
    return;
  }
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int i = 0; i < od; ++i) ss = __fadd_rn(ss, __fmul_rn(pooled[i], pooled[i]));
    s_norm = ss == 0.0f ? 0.0f : (float)sqrt((double)ss);
  }
  __syncthreads();
  float nrm = s_norm;
  float* dst = out + out_offsets[s];
  for (int i = threadIdx.x; i < od; i += blockDim.x) dst[i] = nrm == 0.0f ? pooled[i] : __fdiv_rn(pooled[i], nrm);
}

// One CTA per row: QuantizeSymmetricINT8Into (quantize.go:29-69) of the row
// as one buffer: absmax, scale = absmax / 127, codes of the exact product.
__global__ void quantize_rows_kernel(const float* __restrict__ x, int K, uint32_t* __restrict__ absmax,
                                     __half* __restrict__ codes) {
  __shared__ float s_red[32];
  const int row = blockIdx.x;
  const float* xr = x + (int64_t)row * K;
  float m = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(xr[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) s_red[0] = v;
  }
  __syncthreads();
  const uint32_t bits = __float_as_uint(s_red[0]);
  if (threadIdx.x == 0) absmax[row] = bits;
  float sc, inv;
  seq_scale_ref(bits, &sc, &inv);
  for (int i = 4 * threadIdx.x; i < K; i += 4 * blockDim.x) {
    const uint2 c = quant_codes4(*reinterpret_cast<const float4*>(xr + i), inv);
    *reinterpret_cast<uint2*>(codes + (int64_t)row * K + i) = c;
  }
}

// l2Normalize (model.go:808-820) of a row prefix: float32 sum of squares in
// order, v / float32(sqrt(float64(sum))), unchanged when the sum is 0.
__global__ void l2_rows_kernel(const float* __restrict__ x, int K, const int32_t* __restrict__ out_dims,
                               const int64_t* __restrict__ out_offsets, float* __restrict__ out) {
  __shared__ float s_norm;
  const int row = blockIdx.x, od = out_dims[row];
  const float* xr = x + (int64_t)row * K;
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int i = 0; i < od; ++i) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
    s_norm = ss == 0.0f ? 0.0f : (float)sqrt((double)ss);
  }
  __syncthreads();
  const float nrm = s_norm;
  float* dst = out + out_offsets[row];
  for (int i = threadIdx.x; i < od; i += blockDim.x) dst[i] = nrm == 0.0f ? xr[i] : __fdiv_rn(xr[i], nrm);
}

cudaError_t launch_quantize_rows(const float* x, int rows, int K, uint32_t* absmax, __half* codes,
                                 cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (K % 4 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(codes) & 7))
    return cudaErrorInvalidValue;
  quantize_rows_kernel<<<rows, 256, 0, stream>>>(x, K, absmax, codes);
  return cudaGetLastError();
}

cudaError_t launch_l2_rows(const float* x, int rows, int K, const int32_t* out_dims, const int64_t* out_offsets,
                           float* out, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  l2_rows_kernel<<<rows, 256, 0, stream>>>(x, K, out_dims, out_offsets, out);
  return cudaGetLastError();
}

cudaError_t launch_pool_l2(const float* hidden, const float* inv_rms, const float* w, int H, SeqMeta meta,
                           const int32_t* out_dims, const int64_t* out_offsets, float* out, cudaStream_t stream) {
  if (meta.B == 0) return cudaSuccess;
  pool_l2_kernel<<<meta.B, 256, H * sizeof(float), stream>>>(hidden, inv_rms, w, H, meta, out_dims, out_offsets,
                                                             out);
  return cudaGetLastError();
}

}  // namespace sem
