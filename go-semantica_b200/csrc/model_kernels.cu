// Element-wise and row kernels of the EmbeddingGemma forward pass (sm_100a).
//
// Each kernel restates one step of internal/runtime/model_int8.go:148-256 so
// that its float32 results are bit-identical to the reference's Go code:
// the RMSNorm sum of squares follows the 8-lane AVX2 order, multiplies are
// unfused, divisions and square roots are IEEE-rounded (--fmad=false, no
// fast-math). Rows of a batch are packed back to back; row_seq maps a row to
// its sequence, whose activation scale is the absmax of that sequence alone
// (the reference quantises one whole sequence per call, quantize.go:29-69).
#include "common.cuh"
#include "kernels.h"

namespace sem {

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
__global__ void quantize_kernel(const float* __restrict__ x, const float* __restrict__ inv_rms,
                                const float* __restrict__ w, int K, SeqMeta meta,
                                const uint32_t* __restrict__ absmax, __half* __restrict__ codes) {
  int per_row = K / 16;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)meta.T * per_row) return;
  int64_t row = i / per_row;
  int c = (int)(i % per_row) * 16;
  float scale, inv;
  seq_scale_ref(absmax[meta.row_seq ? meta.row_seq[row] : 0], &scale, &inv);
  const float4* xp = reinterpret_cast<const float4*>(x + row * K + c);
  float v[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float4 t = xp[k];
    v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
  }
  if (inv_rms) {
    float r = inv_rms[row];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], r), w[c + k]);
  }
  __align__(16) __half h[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) h[k] = __int2half_rn(quant_code_ref(v[k], inv));
  uint4* dst = reinterpret_cast<uint4*>(codes + row * K + c);
  dst[0] = reinterpret_cast<const uint4*>(h)[0];
  dst[1] = reinterpret_cast<const uint4*>(h)[1];
}

cudaError_t launch_quantize(const float* x, const float* inv_rms, const float* w, int K, SeqMeta meta,
                            const uint32_t* absmax, __half* codes, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  int64_t n = (int64_t)meta.T * (K / 16);
  quantize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, inv_rms, w, K, meta, absmax, codes);
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

__global__ void qk_norm_rope_kernel(const float* __restrict__ qkv, const float* __restrict__ q_norm,
                                    const float* __restrict__ k_norm, const float* __restrict__ rope_cos,
                                    const float* __restrict__ rope_sin, float eps, int nh, SeqMeta meta,
                                    __half* __restrict__ qh, __half* __restrict__ ql, __half* __restrict__ kh,
                                    __half* __restrict__ kl, __half* __restrict__ vh, __half* __restrict__ vl) {
  int lane = threadIdx.x & 31, g = lane >> 3, sub = lane & 7;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int ld = (nh + 2) * kHeadDim;
  for (int64_t row = warp; row < meta.T; row += nwarps) {  // uniform per warp
    const float* base = qkv + row * ld;
    bool active = g <= nh;
    int gh = active ? g : nh;  // inactive groups mirror the k head and store nothing
    const float* x = base + gh * kHeadDim;
    const float* wn = gh < nh ? q_norm : k_norm;
    float ss = row_sumsq_ref(x, kHeadDim, sub);
    float inv = rms_inv_ref(ss, kHeadDim, eps);
    int pos = meta.row_pos[row];
    const float* cs = rope_cos + (int64_t)pos * (kHeadDim / 2);
    const float* sn = rope_sin + (int64_t)pos * (kHeadDim / 2);
    __half* dh = gh < nh ? qh + (row * nh + gh) * kHeadDim : kh + row * kHeadDim;
    __half* dl = gh < nh ? ql + (row * nh + gh) * kHeadDim : kl + row * kHeadDim;
    if (active) {
#pragma unroll 4
      for (int v = 0; v < 16; ++v) {
        int i = 8 * v + sub;
        // the reference skips a head norm whose weight tensor is absent (model_int8.go:374, :408)
        float x0 = wn ? __fmul_rn(__fmul_rn(x[i], inv), wn[i]) : x[i];
        float x1 = wn ? __fmul_rn(__fmul_rn(x[i + 128], inv), wn[i + 128]) : x[i + 128];
        float c = cs[i], s = sn[i];
        float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        __half h, l;
        split_half(r0, h, l);
        dh[i] = h; dl[i] = l;
        split_half(r1, h, l);
        dh[i + 128] = h; dl[i + 128] = l;
      }
    }
    // v: all 32 lanes, 8 consecutive elements each
    const float* vx = base + (nh + 1) * kHeadDim + lane * 8;
    __half hv[8], lv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) split_half(vx[k], hv[k], lv[k]);
    *reinterpret_cast<uint4*>(vh + row * kHeadDim + lane * 8) = *reinterpret_cast<uint4*>(hv);
    *reinterpret_cast<uint4*>(vl + row * kHeadDim + lane * 8) = *reinterpret_cast<uint4*>(lv);
  }
}

cudaError_t launch_qk_norm_rope(const float* qkv, const float* q_norm, const float* k_norm, const float* rope_cos,
                                const float* rope_sin, float eps, int num_heads, SeqMeta meta, __half* qh,
                                __half* ql, __half* kh, __half* kl, __half* vh, __half* vl, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  if (num_heads < 1 || num_heads > 3) return cudaErrorInvalidValue;
  int64_t warps = meta.T;
  int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  qk_norm_rope_kernel<<<(unsigned)blocks, 256, 0, stream>>>(qkv, q_norm, k_norm, rope_cos, rope_sin, eps, num_heads,
                                                            meta, qh, ql, kh, kl, vh, vl);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Post-norm + residual (model_int8.go:202-210, :224-232) fused with the next
// norm's statistics (:194/:216 of the following step, or output_norm :236).
// ---------------------------------------------------------------------------
__global__ void residual_norm_kernel(const float* __restrict__ o, const float* __restrict__ post_w,
                                     float* __restrict__ hidden, const float* __restrict__ next_w, int H, float eps,
                                     SeqMeta meta, float* __restrict__ inv_rms, uint32_t* __restrict__ absmax) {
  int lane = threadIdx.x & 31, sub = lane & 7;
  int64_t group = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  int64_t ngroups = ((int64_t)gridDim.x * blockDim.x) >> 3;
  int64_t rounds = ((int64_t)meta.T + ngroups - 1) / ngroups;
  for (int64_t it = 0; it < rounds; ++it) {
    int64_t row = group + it * ngroups;
    bool valid = row < meta.T;
    int64_t rr = valid ? row : 0;
    const float* orow = o + rr * H;
    float* hrow = hidden + rr * H;
    float inv1 = rms_inv_ref(row_sumsq_ref(orow, H, sub), H, eps);
    // new hidden and its sum of squares in the same 8-lane order
    float acc = 0.0f;
    for (int v = 0; v < H / 8; ++v) {
      int e = 8 * v + sub;
      // an absent post-norm leaves o as it is (model_int8.go:203, :225)
      float ov = post_w ? __fmul_rn(__fmul_rn(orow[e], inv1), post_w[e]) : orow[e];
      float nv = __fadd_rn(ov, hrow[e]);
      if (valid) hrow[e] = nv;
      acc = fmaf(nv, nv, acc);
    }
    const unsigned full = 0xffffffffu;
    float hi = __shfl_down_sync(full, acc, 4, 8);
    float s = __fadd_rn(acc, hi);
    float s1 = __shfl_down_sync(full, s, 1, 8);
    float p = __fadd_rn(s, s1);
    float p2 = __shfl_down_sync(full, p, 2, 8);
    float tot = __shfl_sync(full, __fadd_rn(p, p2), 0, 8);
    float inv2 = rms_inv_ref(tot, H, eps);
    float m = 0.0f;
    if (absmax) {
      __syncwarp();
      for (int v = 0; v < H / 8; ++v) {
        int e = 8 * v + sub;
        float nv = valid ? hrow[e] : 0.0f;
        m = fmaxf(m, fabsf(__fmul_rn(__fmul_rn(nv, inv2), next_w[e])));
      }
      m = group_max8(m);
    }
    if (valid && sub == 0) inv_rms[row] = inv2;
    if (absmax) warp_seq_atomic_max(absmax, meta.row_seq, valid ? row : -1, m);
  }
}

cudaError_t launch_residual_norm(const float* o, const float* post_w, float* hidden, const float* next_w, int H,
                                 float eps, SeqMeta meta, float* inv_rms, uint32_t* absmax, cudaStream_t stream) {
  if (meta.T == 0) return cudaSuccess;
  residual_norm_kernel<<<row_grid(meta.T), 256, 0, stream>>>(o, post_w, hidden, next_w, H, eps, meta, inv_rms,
                                                             absmax);
  return cudaGetLastError();
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
  int od = out_dims[s];
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

cudaError_t launch_pool_l2(const float* hidden, const float* inv_rms, const float* w, int H, SeqMeta meta,
                           const int32_t* out_dims, const int64_t* out_offsets, float* out, cudaStream_t stream) {
  if (meta.B == 0) return cudaSuccess;
  pool_l2_kernel<<<meta.B, 256, H * sizeof(float), stream>>>(hidden, inv_rms, w, H, meta, out_dims, out_offsets,
                                                             out);
  return cudaGetLastError();
}

}  // namespace sem
