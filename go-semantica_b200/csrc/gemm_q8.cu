// Q8_0 weights x INT8 activations (MatMulQ8_0INT8, internal/kernels/quantize.go:346-458).
//
// The reference sums int8 products exactly inside each 32-element Q8_0 block
// and only then applies the block's fp16 scale in float32. One int8 tensor-core
// MMA with K = 32 (mma.m16n8k32.s8) computes exactly one such block sum, so the
// int32 block dot products here are bit-identical to the reference's; the
// float rescale accumulates blocks in order (one accumulator instead of the
// reference's 8 SIMD lanes, so results agree to float32 rounding).
//
// The MMA accumulator is seeded with the bit pattern of 1.5*2^23: for block
// sums |s| < 2^22 the int32 result, read as a float, is exactly 1.5*2^23 + s,
// so converting to float costs one packed add and the rescale one packed FMA
// (f32x2 on sm_100). Tiles: 128x128 outputs, 128-byte K stages (4 Q8_0 blocks),
// 4-stage cp.async pipeline, 8 warps of 64x32.
#include "common.cuh"
#include "kernels.h"

namespace sem {

namespace {
constexpr int BM = 128, BN = 128, BK = 128, STAGES = 4, THREADS = 256;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, S_BYTES = BN * (BK / 32) * 4;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + S_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES;

__device__ __forceinline__ int swz(int r, int c) { return r * BK + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void mma_s8_biased(int* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(kFloatMagicBits));
}
}  // namespace

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q8_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ W, const float* __restrict__ WS, int M,
                   int N, int K, const uint32_t* __restrict__ a_absmax, const int32_t* __restrict__ row_seq,
                   float* __restrict__ C, uint32_t* __restrict__ out_absmax) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm0 = (warp >> 2) * 64, wn0 = (warp & 3) * 32;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nkb = K / 32, KT = K / BK;

  auto load_stage = [&](int stage, int kt) {
    uint8_t* sa = smem + stage * STAGE_BYTES;
    uint8_t* sb = sa + A_BYTES;
    float* ss = reinterpret_cast<float*>(sb + B_BYTES);
    const int k0 = kt * BK;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = tid + i * THREADS;  // 0..1023
      int r = idx >> 3, c = idx & 7;
      bool va = (m0 + r) < M;
      const int8_t* ga = A + (int64_t)(va ? m0 + r : 0) * K + k0 + c * 16;
      cp_async16(sa + swz(r, c), ga, va);
      const int8_t* gb = W + (int64_t)(n0 + r) * K + k0 + c * 16;
      cp_async16(sb + swz(r, c), gb, true);
    }
    if (tid < BN) {
      const float* gs = WS + (int64_t)(n0 + tid) * nkb + kt * (BK / 32);
      cp_async16(ss + tid * 4, gs, true);
    }
  };

  uint64_t acc[4][4][2];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = 0;
  const uint64_t neg_magic = pack2(-kFloatMagic, -kFloatMagic);

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < KT) load_stage(s, s);
    cp_async_commit();
  }

  for (int kt = 0; kt < KT; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    {
      int nk = kt + STAGES - 1;
      if (nk < KT) load_stage(nk % STAGES, nk);
      cp_async_commit();
    }
    const int stage = kt % STAGES;
    const uint8_t* sa = smem + stage * STAGE_BYTES;
    const uint8_t* sb = sa + A_BYTES;
    const float* ss = reinterpret_cast<const float*>(sb + B_BYTES);
#pragma unroll
    for (int kb = 0; kb < BK / 32; ++kb) {
      const int c0 = kb * 2;
      uint32_t a[4][4], b[4][2];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        int r = wm0 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int c = c0 + (lane >> 4);
        ldmatrix_x4(a[mt][0], a[mt][1], a[mt][2], a[mt][3], sa + swz(r, c));
      }
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        int r = wn0 + p * 16 + (lane & 7) + (lane >> 4) * 8;
        int c = c0 + ((lane >> 3) & 1);
        ldmatrix_x4(b[2 * p][0], b[2 * p][1], b[2 * p + 1][0], b[2 * p + 1][1], sb + swz(r, c));
      }
      uint64_t sc[4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        int col = wn0 + nt * 8 + (lane & 3) * 2;
        sc[nt] = pack2(ss[col * 4 + kb], ss[(col + 1) * 4 + kb]);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          int d[4];
          mma_s8_biased(d, a[mt], b[nt]);
          uint64_t f01 = add2(pack2(__int_as_float(d[0]), __int_as_float(d[1])), neg_magic);
          uint64_t f23 = add2(pack2(__int_as_float(d[2]), __int_as_float(d[3])), neg_magic);
          acc[mt][nt][0] = fma2(f01, sc[nt], acc[mt][nt][0]);
          acc[mt][nt][1] = fma2(f23, sc[nt], acc[mt][nt][1]);
        }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the pipeline buffers are reused below for the row maxima
  float* s_rowmax = reinterpret_cast<float*>(smem);  // [BM][4 column groups]

  // ---- epilogue: dst = sum * inputScale (quantize.go:453) ----
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = m0 + wm0 + mt * 16 + g + h * 8;
      const bool valid = row < M;
      float rs = 0.0f;
      if (valid) {
        float inv;
        seq_scale_ref(a_absmax[row_seq ? row_seq[row] : 0], &rs, &inv);
      }
      if (EPI == kEpiStore) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          float v0, v1;
          unpack2(acc[mt][nt][h], v0, v1);
          const int col = n0 + wn0 + nt * 8 + t4 * 2;
          if (valid)
            *reinterpret_cast<float2*>(C + (int64_t)row * N + col) = make_float2(__fmul_rn(v0, rs), __fmul_rn(v1, rs));
        }
      } else {
        // runMLPINT8 (model_int8.go:523-530): gate and up scaled, GELUQuick(gate) * up
        float mm = 0.0f;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          float g0, g1, u0, u1;
          unpack2(acc[mt][2 * p][h], g0, g1);
          unpack2(acc[mt][2 * p + 1][h], u0, u1);
          const float h0 = __fmul_rn(gelu_quick_ref(__fmul_rn(g0, rs)), __fmul_rn(u0, rs));
          const float h1 = __fmul_rn(gelu_quick_ref(__fmul_rn(g1, rs)), __fmul_rn(u1, rs));
          const int ch = ((n0 + wn0) >> 1) + p * 8 + t4 * 2;
          if (valid) *reinterpret_cast<float2*>(C + (int64_t)row * (N / 2) + ch) = make_float2(h0, h1);
          mm = fmaxf(mm, fmaxf(fabsf(h0), fabsf(h1)));
        }
        // per-row max over the 4 lanes of the quad (all lanes participate)
        mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, 1));
        mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, 2));
        if (t4 == 0) s_rowmax[(wm0 + mt * 16 + g + h * 8) * 4 + (warp & 3)] = valid ? mm : 0.0f;
      }
    }
  if (EPI == kEpiGeluUp && out_absmax) {
    // One atomic per CTA when the tile's rows share a sequence (the usual
    // case); per-row atomics only on tiles that straddle sequences.
    __syncthreads();
    const int last = min(m0 + BM, M) - 1;
    const int seq0 = row_seq ? row_seq[m0] : 0;
    const bool uniform = !row_seq || row_seq[last] == seq0;
    float rmax = 0.0f;
    const int r = tid;
    if (r < BM) {
      rmax = fmaxf(fmaxf(s_rowmax[r * 4], s_rowmax[r * 4 + 1]), fmaxf(s_rowmax[r * 4 + 2], s_rowmax[r * 4 + 3]));
      if (!uniform && m0 + r < M) atomicMax(&out_absmax[row_seq[m0 + r]], __float_as_uint(rmax));
    }
    if (uniform) {
      rmax = warp_max(rmax);
      __syncthreads();
      if (lane == 0) s_rowmax[warp] = rmax;
      __syncthreads();
      if (tid == 0) {
        float m = s_rowmax[0];
        for (int w = 1; w < THREADS / 32; ++w) m = fmaxf(m, s_rowmax[w]);
        atomicMax(&out_absmax[seq0], __float_as_uint(m));
      }
    }
  }
}

cudaError_t launch_gemm_q8(const int8_t* a_codes, const int8_t* w_codes, const float* w_scales, int M, int N, int K,
                           const uint32_t* a_absmax, const int32_t* row_seq, float* c, int epilogue,
                           uint32_t* out_absmax, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (N % BN != 0 || K % BK != 0) return cudaErrorInvalidValue;
  dim3 grid(N / BN, (M + BM - 1) / BM);
  // the attribute is per device context: set it on every launch (cheap host call)
  if (epilogue == kEpiStore) {
    cudaFuncSetAttribute(gemm_q8_kernel<kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    gemm_q8_kernel<kEpiStore><<<grid, THREADS, SMEM_BYTES, stream>>>(a_codes, w_codes, w_scales, M, N, K, a_absmax,
                                                                     row_seq, c, out_absmax);
  } else {
    cudaFuncSetAttribute(gemm_q8_kernel<kEpiGeluUp>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    gemm_q8_kernel<kEpiGeluUp><<<grid, THREADS, SMEM_BYTES, stream>>>(a_codes, w_codes, w_scales, M, N, K, a_absmax,
                                                                      row_seq, c, out_absmax);
  }
  return cudaGetLastError();
}

}  // namespace sem
