// Q8_0 x INT8 projection on CUDA cores in the reference's VNNI lane order
// (internal/kernels/simd_amd64.s:241-304, matmulInnerLoopVNNIAsm, and
// quantize.go:390-458, matMulQ8_0INT8SerialRange):
//
//   for each 32-element block kb:   lane l (0..7) gets the exact int32 sum of
//     the 4 products of bytes 4l..4l+3 (VPDPBUSD with the zero-point
//     correction), converted to float32 and fused-multiply-added with the
//     block's scale into the lane's float32 accumulator (VFMADD231PS);
//   sum = ((l0 + l4) + (l1 + l5)) + ((l2 + l6) + (l3 + l7))   (VEXTRACTF128,
//     VADDPS, VHADDPS, VHADDPS);
//   dst = sum * inputScale                                     (unfused).
//
// Every output is therefore bit-identical to the reference's default amd64
// build on an AVX512-VNNI host. This is the kernel for small batches and for
// sequences shorter than 128 tokens: no tensor-core pipeline to fill, no TMEM
// drain, and the reference's exact float32 order.
//
// Mapping: the 8 lane accumulators of one output live in 8 consecutive threads
// (a "group"); the horizontal sum is three xor shuffles inside the group, in
// the order above (float addition is commutative, so both partners of every
// shuffle hold the same bits). A group owns a register tile of 4 tokens x 4
// weight rows. The 4-byte partial is one dp4a whose accumulator input is the
// bit pattern of 1.5 * 2^23, so its result read as a float is 1.5 * 2^23 +
// partial exactly (|partial| <= 4 * 127 * 127 < 2^22) and one exact subtraction
// gives float32(partial) without a conversion instruction.
//
// Data: activation codes arrive as fp16 integers (the tensor-core kernels'
// operand type) and are packed to int8 while staged into shared memory; the
// weights use an int8 plane whose rows are stored lane-major ([lane][block]
// words), so a thread reads four consecutive blocks of its lane with one
// 16-byte shared-memory load; block scales are the runtime f16 decoder's fp32
// values (model_int8.go:543-597).
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace sem {
namespace {

constexpr int kDpThreads = 256;  // 32 groups of 8 lane threads
constexpr int kDpStages = 3;     // weight-chunk ring
constexpr int kDpChunk = 12;     // blocks per weight chunk (K % 384 == 0), else 4
constexpr int kDpCtasPerSm = 2;

// Words between the lanes of one row in shared memory: a multiple of 4 whose
// quarter is odd, so the 8 lanes of a group read 8 different bank quads.
__host__ __device__ constexpr int dp_lane_stride(int blocks) { return ((blocks / 4) & 1) ? blocks : blocks + 4; }
__host__ __device__ constexpr int dp_chunk(int kb_total) { return kb_total % kDpChunk == 0 ? kDpChunk : 4; }

// 8 INT8 codes held as fp16 integers in [-127, 127] -> two words of int8.
// h + 1152 lies in [1025, 1279], where fp16 steps by 1, so the low byte of its
// bit pattern is h + 128; xor 0x80 gives the two's complement byte of h.
__device__ __forceinline__ uint2 codes8_to_s8(uint4 v) {
  const __half2 mg = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t t[4];
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __hadd2(*reinterpret_cast<const __half2*>(&w[i]), mg);
    t[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint2(__byte_perm(t[0], t[1], 0x6420) ^ 0x80808080u, __byte_perm(t[2], t[3], 0x6420) ^ 0x80808080u);
}

// One lane's block term: acc = fma(float32(exact 4-byte partial), scale,
// acc). The dp4a accumulator input 1.5 * 2^23 makes the result's float bits
// 1.5 * 2^23 + partial, and subtracting 1.5 * 2^23 is exact. dp4a runs on the
// heavy FMA pipe at half rate; the scalar subtraction and FMA can issue on
// either FMA pipe (packed f32x2 forms measured slower).
__device__ __forceinline__ float lane_fma(uint32_t a, uint32_t w, float s, float acc) {
  const float x = __int_as_float(__dp4a((int)a, (int)w, kFloatMagicBits));
  return __fmaf_rn(__fsub_rn(x, kFloatMagic), s, acc);
}

// The VNNI kernel's horizontal sum over the 8 threads of a group; every
// thread of the group receives the same bits.
__device__ __forceinline__ float group_hsum(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));  // l + (l ^ 4)
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));  // (l0+l4) + (l1+l5), (l2+l6) + (l3+l7)
  return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// GELUQuick(gate * rs) * (up * rs) (model_int8.go:523-530).
__device__ __forceinline__ float dp_gelu_up(float g, float u, float rs) {
  return __fmul_rn(gelu_quick_ref(__fmul_rn(g, rs)), __fmul_rn(u, rs));
}

// TGM token groups x (32 / TGM) weight-row groups per tile: TM = 4 TGM tokens,
// TN = 4 (32 / TGM) weight rows. A CTA stages its TM tokens' codes once (all
// of K) and walks the weight tiles blockIdx.x, blockIdx.x + gridDim.x, ...;
// the weights stream through a kDpStages-deep ring of (tile, K chunk) items.
// kEpiGeluUp: a group's 4 rows are gate j, j + 1 and up j, j + 1, so it forms
// two outputs h = GELUQuick(gate) * up per token, and the CTA the per-sequence
// absmax of h over all its tiles.
// KBT: the blocks per row (K / 32) when known at compile time (the model's
// K = 768, 1152 and 3072), so the shared-memory strides fold into the load
// instructions; 0 takes K at run time.
template <int TGM, int EPI, int KBT>
__global__ void __launch_bounds__(kDpThreads, kDpCtasPerSm) gemm_q8_dp4a_kernel(
    const __half* __restrict__ a, const uint32_t* __restrict__ wl, const float* __restrict__ ws, int M, int N, int K,
    const uint32_t* __restrict__ a_absmax, const int32_t* __restrict__ row_seq, float* __restrict__ c,
    uint32_t* __restrict__ out_absmax) {
  constexpr int TM = 4 * TGM, TN = 4 * (32 / TGM);
  extern __shared__ __align__(16) uint32_t dp_smem[];
  __shared__ float s_rs[TM];
  __shared__ int s_seq[TM];
  __shared__ uint32_t s_amax[TM];
  const int KB = KBT > 0 ? KBT : K / 32, KW = 8 * KB;  // blocks and words per row
  const int kbc = dp_chunk(KB), pieces = kbc / 4, nchunks = KB / kbc;
  const int la = dp_lane_stride(KB), lw = dp_lane_stride(kbc);
  uint32_t* As = dp_smem;                // [TM][8][la] activation words, all of K
  uint32_t* ring = As + TM * 8 * la;     // stages of {weights [TN][8][lw] words, scales [TN][lw]}
  const int stage_words = TN * 8 * lw + TN * lw;
  const int tid = threadIdx.x, l = tid & 7, g = tid >> 3;
  const int tg = g % TGM, cg = g / TGM;
  const int m0 = blockIdx.y * TM;
  const int n_tiles = N / TN;
  const int my_tiles = (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int items = my_tiles * nchunks;
  const int half = N / 2;  // kEpiGeluUp: gate rows [0, half), up rows [half, N)
  auto wrow = [&](int nt, int slot) -> int {
    if (EPI == kEpiStore) return nt * TN + slot;
    const int q = slot & 3;
    const int j = nt * (TN / 2) + 2 * (slot >> 2) + (q & 1);
    return q < 2 ? j : half + j;
  };
  // This thread's share of every item's copies is the same list of (shared
  // offset, global offset) pairs, shifted per item by the weight tile and the
  // K chunk: computed once here (a weight tile's rows move by TN rows per
  // tile, or TN / 2 gate and up rows each under kEpiGeluUp).
  constexpr int kMaxW = (TN * 8 * 3 + kDpThreads - 1) / kDpThreads;  // pieces <= 3
  const int64_t tile_rows = EPI == kEpiStore ? TN : TN / 2;
  int w_soff[kMaxW], w_goff[kMaxW];  // word offsets (a weight plane holds < 2^31 words)
  int n_w = 0;
#pragma unroll
  for (int k = 0; k < kMaxW; ++k) {
    const int i = tid + k * kDpThreads;
    w_soff[k] = 0;
    w_goff[k] = 0;
    if (i < TN * 8 * pieces) {
      const int p = i % pieces, rest = i / pieces, ll = rest & 7, slot = rest >> 3;
      w_soff[k] = (slot * 8 + ll) * lw + 4 * p;
      w_goff[k] = wrow(0, slot) * KW + ll * KB + 4 * p;
      n_w = k + 1;
    }
  }
  int s_soff = -1, s_goff = 0;
  if (tid < TN * pieces) {
    const int p = tid % pieces, slot = tid / pieces;
    s_soff = slot * lw + 4 * p;
    s_goff = wrow(0, slot) * KB + 4 * p;
  }
  // one (tile, chunk) item's weights and block scales into its stage;
  // every thread commits a group per call (empty past the end) so the wait
  // counts stay uniform
  auto issue = [&](int item) {
    if (item < items) {
      const int tix = item / nchunks, kc0 = (item - tix * nchunks) * kbc;
      const int64_t nt = (int64_t)blockIdx.x + (int64_t)tix * gridDim.x;
      uint32_t* Ws = ring + (item % kDpStages) * stage_words;
      float* Ss = reinterpret_cast<float*>(Ws + TN * 8 * lw);
      const uint32_t* wsrc = wl + nt * tile_rows * KW + kc0;
#pragma unroll
      for (int k = 0; k < kMaxW; ++k)
        if (k < n_w) cp_async16(Ws + w_soff[k], wsrc + w_goff[k], true);
      if (s_soff >= 0) cp_async16(Ss + s_soff, ws + nt * tile_rows * KB + kc0 + s_goff, true);
    }
    cp_async_commit();
  };
  for (int i = 0; i < kDpStages - 1; ++i) issue(i);

  if (tid < TM) {
    const int m = m0 + tid;
    int sq = -1;
    float rs = 0.0f, inv;
    if (m < M) {
      sq = row_seq ? row_seq[m] : 0;
      seq_scale_ref(a_absmax[sq], &rs, &inv);
    }
    s_seq[tid] = sq;
    s_rs[tid] = rs;
    s_amax[tid] = 0u;
  }
  // activation codes: fp16 -> int8 words, lane-major, loads batched 4 deep
  {
    const int n = TM * KB * 4;  // 16-byte pieces of 8 codes
    for (int i0 = tid; i0 < n; i0 += 4 * kDpThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kDpThreads;
        const int h = i & 3, kb = (i >> 2) % KB, t = (i >> 2) / KB;
        v[u] = make_uint4(0x3c003c00u, 0u, 0u, 0u);
        if (i < n && m0 + t < M)
          v[u] = *reinterpret_cast<const uint4*>(a + (size_t)(m0 + t) * K + (size_t)kb * 32 + 8 * h);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kDpThreads;
        if (i >= n) break;
        const int h = i & 3, kb = (i >> 2) % KB, t = (i >> 2) / KB;
        const uint2 wd = m0 + t < M ? codes8_to_s8(v[u]) : make_uint2(0u, 0u);
        As[(t * 8 + 2 * h) * la + kb] = wd.x;
        As[(t * 8 + 2 * h + 1) * la + kb] = wd.y;
      }
    }
  }

  float acc[4][4];  // 4 tokens x 4 weight rows
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q] = 0.0f;

  for (int it = 0; it < items; ++it) {
    cp_async_wait<kDpStages - 2>();  // this thread's copies of item `it` have landed
    // item `it` (and, the first time, the activation codes) visible to all;
    // every thread is past item it - 1, so its stage takes item it + kDpStages - 1
    __syncthreads();
    issue(it + kDpStages - 1);
    const uint32_t* Ws = ring + (it % kDpStages) * stage_words;
    const float* Ss = reinterpret_cast<const float*>(Ws + TN * 8 * lw);
    const int kc0 = (it % nchunks) * kbc;
#pragma unroll
    for (int p = 0; p < pieces; ++p) {
      uint4 av[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
        av[r] = *reinterpret_cast<const uint4*>(As + ((tg * 4 + r) * 8 + l) * la + kc0 + 4 * p);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int slot = cg * 4 + q;
        const uint4 wv = *reinterpret_cast<const uint4*>(Ws + (slot * 8 + l) * lw + 4 * p);
        const float4 sv = *reinterpret_cast<const float4*>(Ss + slot * lw + 4 * p);
        // blocks 4p .. 4p + 3 of the chunk, in ascending order per accumulator
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          acc[r][q] = lane_fma(av[r].x, wv.x, sv.x, acc[r][q]);
          acc[r][q] = lane_fma(av[r].y, wv.y, sv.y, acc[r][q]);
          acc[r][q] = lane_fma(av[r].z, wv.z, sv.z, acc[r][q]);
          acc[r][q] = lane_fma(av[r].w, wv.w, sv.w, acc[r][q]);
        }
      }
    }
    if (it % nchunks == nchunks - 1) {  // the tile's last chunk: its epilogue
      const int nt = (int)blockIdx.x + (it / nchunks) * (int)gridDim.x;
      float v[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[r][q] = acc[r][q];
          acc[r][q] = 0.0f;
        }
      if (EPI == kEpiStore) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int t = tg * 4 + r, m = m0 + t;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float sum = group_hsum(v[r][q]);
            if (((r * 4 + q) & 7) == l && m < M) c[(size_t)m * N + nt * TN + cg * 4 + q] = __fmul_rn(sum, s_rs[t]);
          }
        }
      } else {
        // lane l: token r = l / 2, channel j + (l & 1)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float g0 = group_hsum(v[r][0]), g1 = group_hsum(v[r][1]);
          const float u0 = group_hsum(v[r][2]), u1 = group_hsum(v[r][3]);
          const int t = tg * 4 + r, m = m0 + t;
          if ((l >> 1) == r && m < M) {
            const float h = dp_gelu_up((l & 1) ? g1 : g0, (l & 1) ? u1 : u0, s_rs[t]);
            c[(size_t)m * half + nt * (TN / 2) + cg * 2 + (l & 1)] = h;
            const float am = fmaxf(0.0f, fabsf(h));  // NaN folds to 0, as fmaxf does in the tensor-core epilogues
            if (out_absmax && am > 0.0f) atomicMax(&s_amax[t], __float_as_uint(am));
          }
        }
      }
    }
  }
  __syncthreads();  // every epilogue's shared absmax updates are in
  if (EPI == kEpiGeluUp && out_absmax && tid < TM && s_seq[tid] >= 0 && s_amax[tid])
    atomicMax(&out_absmax[s_seq[tid]], s_amax[tid]);
}

template <int TGM, int EPI, int KBT>
cudaError_t launch_dp(const __half* a, const int8_t* wl, const float* ws, int M, int N, int K, const uint32_t* a_absmax,
                      const int32_t* row_seq, float* c, uint32_t* out_absmax, cudaStream_t stream) {
  constexpr int TM = 4 * TGM, TN = 4 * (32 / TGM);
  const int KB = K / 32, kbc = dp_chunk(KB);
  const size_t smem =
      ((size_t)TM * 8 * dp_lane_stride(KB) + (size_t)kDpStages * (TN * 8 + TN) * dp_lane_stride(kbc)) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;  // K up to 3072 fits
  auto kern = gemm_q8_dp4a_kernel<TGM, EPI, KBT>;
  int sms = 148;
  {  // per-device: the shared-memory limit (a function attribute) and the SM count
    static std::mutex mu;
    static bool done[64] = {};
    static int sm_count[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
      if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) != cudaSuccess)
        return e;
      if ((e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
      done[dev] = true;
    }
    sms = sm_count[dev];
  }
  // token tiles x weight-tile groups ~ the resident CTAs; each CTA takes
  // ceil(n_tiles / groups) weight tiles, so the activation codes are staged
  // once per that many tiles
  const int m_tiles = (M + TM - 1) / TM, n_tiles = N / TN;
  const int want = (kDpCtasPerSm * sms) / m_tiles;  // at most one wave of CTAs
  const int per = (n_tiles + (want < 1 ? 1 : want) - 1) / (want < 1 ? 1 : want);
  const int gx = (n_tiles + per - 1) / per;
  const dim3 grid((unsigned)gx, (unsigned)m_tiles);
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  kern<<<grid, kDpThreads, smem, stream>>>(a, reinterpret_cast<const uint32_t*>(wl), ws, M, N, K, a_absmax, row_seq, c,
                                           out_absmax);
  return cudaGetLastError();
}

// Calls f with std::integral_constant<int, K / 32> for the model's K values,
// else with 0 (K at run time).
template <class F>
cudaError_t dispatch_dp(int K, F&& f) {
  switch (K) {
    case 768: return f(std::integral_constant<int, 24>{});
    case 1152: return f(std::integral_constant<int, 36>{});
    case 3072: return f(std::integral_constant<int, 96>{});
    default: return f(std::integral_constant<int, 0>{});
  }
}

}  // namespace

cudaError_t launch_gemm_q8_dp4a(const __half* a_codes, const int8_t* w_lanes, const float* w_scales, int M, int N,
                                int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c, int epilogue,
                                uint32_t* out_absmax, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (M < 0 || K <= 0 || K % 128 || N <= 0 || N % 128 || !a_codes || !w_lanes || !w_scales || !a_absmax || !c)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a_codes) | reinterpret_cast<uintptr_t>(w_lanes) |
       reinterpret_cast<uintptr_t>(w_scales)) & 15)
    return cudaErrorMisalignedAddress;
  // 32-token x 16-row tiles (measured 5-9 % faster than 16 x 32 at 512
  // tokens; below 17 tokens they give twice as many CTAs)
  return dispatch_dp(K, [&](auto kbt) {
    constexpr int KBT = decltype(kbt)::value;
    if (epilogue == kEpiGeluUp)
      return launch_dp<8, kEpiGeluUp, KBT>(a_codes, w_lanes, w_scales, M, N, K, a_absmax, row_seq, c, out_absmax,
                                           stream);
    return launch_dp<8, kEpiStore, KBT>(a_codes, w_lanes, w_scales, M, N, K, a_absmax, row_seq, c, nullptr, stream);
  });
}

// Q8_0 blocks of `rows` x `cols` -> the int8 plane of the CUDA-core kernel:
// row r at dst + (dst_row_offset + r) * cols, word (lane * nb + block) holding
// bytes 4 lane .. 4 lane + 3 of that block.
__global__ void repack_q8_0_lanes_kernel(const uint8_t* __restrict__ raw, int64_t rows, int nb,
                                         uint32_t* __restrict__ dst, int64_t dst_row_offset) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one (row, block)
  if (i >= rows * nb) return;
  const int64_t r = i / nb;
  const int b = (int)(i % nb);
  const uint8_t* q = raw + i * 34 + 2;
  uint32_t* row = dst + (dst_row_offset + r) * (int64_t)nb * 8;
#pragma unroll
  for (int l = 0; l < 8; ++l)
    row[l * nb + b] = (uint32_t)q[4 * l] | ((uint32_t)q[4 * l + 1] << 8) | ((uint32_t)q[4 * l + 2] << 16) |
                      ((uint32_t)q[4 * l + 3] << 24);
}

cudaError_t launch_repack_q8_0_lanes(const uint8_t* raw, int64_t rows, int cols, int8_t* dst, int64_t dst_row_offset,
                                     cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (cols % 32 || (reinterpret_cast<uintptr_t>(dst) & 3)) return cudaErrorInvalidValue;
  const int nb = cols / 32;
  const int64_t n = rows * nb;
  repack_q8_0_lanes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(raw, rows, nb,
                                                                            reinterpret_cast<uint32_t*>(dst),
                                                                            dst_row_offset);
  return cudaGetLastError();
}

}  // namespace sem
