// Q8_0 x INT8 projection for large token counts on the sm_100a tensor cores,
// with the Q8_0 block scales folded into the weights.
//
// The reference (matmulQ8_0INT8*, quantize.go:401-455) sums each 32-element
// block's int8 products exactly and scales the block sum by the block's fp16
// scale in float32. A kernel that keeps each block separate must drain TMEM
// after every 32-wide K step. Here each weight element instead becomes its
// exact value w = q * d (an int8 times an fp16, 18 significant bits) times a
// per-row power of two 2^S_n that puts the row's largest |w| in [2^13, 2^14),
// stored as two fp16 planes hi = fp16(w * 2^S_n) and lo = fp16(w * 2^S_n - hi)
// (hi + lo == w * 2^S_n exactly whenever lo stays a normal fp16, i.e. for any
// block scale within 2^20 of the row's largest). Two kind::f16 MMAs per K
// step (hi, then lo, into the same fp32 TMEM accumulator) give
// sum_k a_k * w_k * 2^S_n with every product exact; only the float32 summation
// order differs from the reference's (within the reference's own spread
// between its builds). The accumulator stays in TMEM for the whole K, so the
// epilogue runs once per tile: out = (acc * 2^-S_n) * inputScale
// (quantize.go:453), the power of two being exact.
//
// QKV, O and down (kEpiStore): the weight rows are the MMA's M = 128 (TMEM
// lanes), 256 tokens are N, one 256-column accumulator per tile, three 64 KB
// stages (hi, lo, tokens). Gate/up (gemm_q8_gateup_kernel): tokens are M and
// the gate and up rows of 128 channels together are N = 256. TMEM holds two
// tiles' accumulators (512 columns) so the epilogue of tile i overlaps the
// MMAs of tile i+1. One persistent CTA per SM: warps 0 and 2 issue TMA for
// alternate stages, warp 1 the MMAs, warps 4-11 (two per TMEM lane quarter)
// the epilogue.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.h"

namespace sem {

namespace {

constexpr int kXK = 64;                 // K elements per stage: 128 bytes of fp16 per row
constexpr int kXM = 128;                // weight rows per tile (TMEM lanes)
constexpr int kXWTile = kXM * kXK * 2;  // 16 KB: one weight plane tile of one stage
constexpr int kXThreads = 384;
constexpr int kXEpiWarps = 8;
constexpr int kXBarBytes = 256;

template <int EPI>
struct XCfg;
template <>
struct XCfg<kEpiStore> {
  static constexpr int NA = 1, NT = 256, STAGES = 3;
};

template <int EPI>
struct XLayout {
  using C = XCfg<EPI>;
  static constexpr int kStage = C::NA * 2 * kXWTile + C::NT * kXK * 2;  // also the TMA transaction count
  static constexpr int kBufCols = C::NA * C::NT;                        // TMEM columns of one tile
  static constexpr int kSmem = 1024 + C::STAGES * kStage + kXBarBytes + 2 * C::NT * 8;
  static_assert(2 * kBufCols <= 512, "two tiles' accumulators must fit TMEM");
  static_assert(kSmem <= 232448, "shared memory per CTA");
  static_assert(C::NT % 32 == 0 && C::NT <= 256, "token tile: two halves of whole 16-column chunks");
};

__device__ uint32_t g_split_error;  // error bits of launches given no error word

// GELUQuick(gate * rs) * (up * rs), the runMLPINT8 element (model_int8.go:523-530).
__device__ __forceinline__ float gelu_up_f(float g, float u, float rs) {
  return __fmul_rn(gelu_quick_ref(__fmul_rn(g, rs)), __fmul_rn(u, rs));
}

}  // namespace

template <int EPI>
__global__ void __launch_bounds__(kXThreads, 1)
    gemm_q8_split_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a, const float* __restrict__ row_scale, int n_per_a,
                         int T, int K, const uint32_t* __restrict__ a_absmax, const int32_t* __restrict__ row_seq,
                         float* __restrict__ c_out, uint32_t* __restrict__ out_absmax, uint32_t* __restrict__ err) {
  using Cf = XCfg<EPI>;
  using L = XLayout<EPI>;
  constexpr int NA = Cf::NA, NT = Cf::NT, ST = Cf::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * L::kStage);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_rs = reinterpret_cast<float*>(smem + ST * L::kStage + kXBarBytes);  // [2][NT]
  static_assert((2 * ST + 5) * 8 + 8 <= kXBarBytes, "barrier block");
  if (!err) err = &g_split_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mt = n_per_a / kXM;
  const int total = n_mt * ((T + NT - 1) / NT);
  const int nks = K / kXK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kXEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers (alternate stages) ----------------
    if (lane == 0) {
      const uint32_t me = warp >> 1;
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_a);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        const int tt = tile / n_mt, mt = tile % n_mt;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          if ((it & 1) != me) continue;
          const uint32_t s = it % ST, u = it / ST;
          if (!mbar_wait(&empty[s], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + s * L::kStage;
          mbar_arrive_expect_tx(&full[s], L::kStage);
#pragma unroll
          for (int a = 0; a < NA; ++a)  // hi then lo rows of the tile: one 3-D copy
            tma_load_3d(&tm_w, &full[s], st + (2 * a) * kXWTile, ks * kXK, a * n_per_a + mt * kXM, 0);
          tma_load_2d(&tm_a, &full[s], st + 2 * NA * kXWTile, ks * kXK, tt * NT);
        }
      }
      // copies in flight land before the CTA's shared memory is released;
      // `it` is one past the last iteration this thread issued or skipped
      for (uint32_t j = it > (uint32_t)ST ? it - ST : 0; j < it; ++j)
        if ((j & 1) == me) mbar_wait_drain(&full[j % ST], (j / ST) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(kXM, NT);
      uint32_t it = 0, tix = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++tix) {
        const uint32_t b = tix & 1, ub = tix >> 1;
        if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + b * L::kBufCols;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const uint32_t s = it % ST, u = it / ST;
          if (!mbar_wait(&full[s], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sw = smem_u32(stages + s * L::kStage);
          const uint32_t sb = sw + 2 * NA * kXWTile;
#pragma unroll
          for (int kk = 0; kk < kXK / 16; ++kk) {
            const uint64_t bdesc = umma_desc_k_sw128(sb + kk * 32);
#pragma unroll
            for (int a = 0; a < NA; ++a) {
              umma_f16(d0 + a * NT, umma_desc_k_sw128(sw + (2 * a) * kXWTile + kk * 32), bdesc, idesc,
                       (ks | kk) ? 1u : 0u);
              umma_f16(d0 + a * NT, umma_desc_k_sw128(sw + (2 * a + 1) * kXWTile + kk * 32), bdesc, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      umma_commit(drain);  // every MMA has finished writing TMEM before it is freed
      mbar_wait_drain(drain, 0);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue ----------------
    constexpr int TPH = NT / 2;  // tokens of a thread's half of the tile
    const int e = warp - 4;
    const int q = warp & 3;      // the TMEM lane quarter this warp may access
    const int half = e >> 2;
    const int etid = e * 32 + lane;
    const int ch = q * 32 + lane;  // weight row (output channel) within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    uint32_t tix = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tix) {
      const int tt = tile / n_mt, mt = tile % n_mt;
      const int t0 = tt * NT;
      const int cur = tix & 1;
      if (etid < NT) {  // per-token input scales of this tile (double-buffered across tiles)
        const int t = t0 + etid;
        const int sq = t < T ? (row_seq ? row_seq[t] : 0) : -1;
        float rs = 0.0f, inv;
        if (sq >= 0) seq_scale_ref(a_absmax[sq], &rs, &inv);
        s_rs[cur * NT + etid] = rs;
      }
      named_bar_sync(1, kXEpiWarps * 32);
      const uint32_t b = tix & 1, ub = tix >> 1;
      if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);  // converged (and agreed) before the .sync.aligned TMEM loads
      if (!ok) continue;
      tc_fence_after();
      const uint32_t tb = t_lane + b * L::kBufCols + half * TPH;
      const float* c_rs = s_rs + cur * NT + half * TPH;
      const int tok0 = t0 + half * TPH;  // first token of this thread's half
      const int n0 = mt * kXM + ch;
      {
        const float rsc = row_scale[n0];
        float* dst = c_out + (size_t)tok0 * n_per_a + n0;
#pragma unroll 1
        for (int c = 0; c < TPH / 16; c += 2) {
          uint32_t r[2][16];
          tmem_ld16(tb + c * 16, r[0]);
          tmem_ld16(tb + c * 16 + 16, r[1]);
          tmem_wait_ld();
          reg_barrier16(r[0]);
          reg_barrier16(r[1]);
          if (c + 2 >= TPH / 16) {  // every value of this tile is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int x = (c + cc) * 16 + i;
              if (tok0 + x < T)  // warp-uniform
                dst[(size_t)x * n_per_a] = __fmul_rn(__fmul_rn(__uint_as_float(r[cc][i]), rsc), c_rs[x]);
            }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Gate/up with the tokens as the MMA's M = 128 (TMEM lanes) and the weights
// as N = 256: 128 gate rows then the 128 up rows of the same channels, so one
// kind::f16 MMA per plane covers both projections (N = 256 MMAs keep the
// tensor pipe far busier than N = 128 ones). The accumulator of a tile holds
// gate in columns [0, 128) and up in [128, 256) for one token per lane, so the
// epilogue forms GELUQuick(gate) * up (runMLPINT8, model_int8.go:510-538) per
// thread, with the channel's row scales from shared memory and the token's
// input scale in a register, and keeps the per-sequence absmax.
constexpr int kGuTok = 128;                     // tokens per tile (TMEM lanes)
constexpr int kGuCh = 128;                      // channels per tile (gate and up rows each)
constexpr int kGuA = kGuTok * kXK * 2;          // 16 KB token tile of a stage
constexpr int kGuB = 2 * kGuCh * kXK * 2;       // 32 KB gate + up rows of one plane
constexpr int kGuStage = kGuA + 2 * kGuB;       // 80 KB
constexpr int kGuStages = 2;
constexpr int kGuSmem = 1024 + kGuStages * kGuStage + kXBarBytes + 2 * 2 * kGuCh * 4;
static_assert(kGuSmem <= 232448, "shared memory per CTA");

__global__ void __launch_bounds__(kXThreads, 1)
    gemm_q8_gateup_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a, const float* __restrict__ row_scale, int F, int T,
                          int K, const uint32_t* __restrict__ a_absmax, const int32_t* __restrict__ row_seq,
                          float* __restrict__ h_out, uint32_t* __restrict__ out_absmax, uint32_t* __restrict__ err) {
  constexpr int ST = kGuStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * kGuStage);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_rsc = reinterpret_cast<float*>(smem + ST * kGuStage + kXBarBytes);  // [2 tiles][gate 128 | up 128]
  if (!err) err = &g_split_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_ct = F / kGuCh;
  const int total = n_ct * ((T + kGuTok - 1) / kGuTok);
  const int nks = K / kXK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kXEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers (alternate stages) ----------------
    if (lane == 0) {
      const uint32_t me = warp >> 1;
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_a);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        const int tt = tile / n_ct, ct = tile % n_ct;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          if ((it & 1) != me) continue;
          const uint32_t s = it % ST, u = it / ST;
          if (!mbar_wait(&empty[s], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + s * kGuStage;
          mbar_arrive_expect_tx(&full[s], kGuStage);
          tma_load_2d(&tm_a, &full[s], st, ks * kXK, tt * kGuTok);
          // [hi, lo][gate, up][128 rows][128 B]: one 4-D copy
          tma_load_4d(&tm_w, &full[s], st + kGuA, ks * kXK, ct * kGuCh, 0, 0);
        }
      }
      for (uint32_t j = it > (uint32_t)ST ? it - ST : 0; j < it; ++j)
        if ((j & 1) == me) mbar_wait_drain(&full[j % ST], (j / ST) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(kGuTok, 2 * kGuCh);
      uint32_t it = 0, tix = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++tix) {
        const uint32_t b = tix & 1, ub = tix >> 1;
        if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + b * (2 * kGuCh);
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const uint32_t s = it % ST, u = it / ST;
          if (!mbar_wait(&full[s], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + s * kGuStage);
#pragma unroll
          for (int kk = 0; kk < kXK / 16; ++kk) {
            const uint64_t adesc = umma_desc_k_sw128(sa + kk * 32);
            umma_f16(d0, adesc, umma_desc_k_sw128(sa + kGuA + kk * 32), idesc, (ks | kk) ? 1u : 0u);
            umma_f16(d0, adesc, umma_desc_k_sw128(sa + kGuA + kGuB + kk * 32), idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      umma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue ----------------
    const int e = warp - 4;
    const int q = warp & 3;     // token lane quarter
    const int half = e >> 2;    // channels [64 half, +64) of the tile
    const int etid = e * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    uint32_t tix = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tix) {
      const int tt = tile / n_ct, ct = tile % n_ct;
      const int cur = tix & 1;
      // the channels' row scales of this tile (double-buffered across tiles)
      s_rsc[cur * 2 * kGuCh + etid] =
          row_scale[(etid < kGuCh ? 0 : F - kGuCh) + ct * kGuCh + etid];  // gate rows, then up rows
      named_bar_sync(1, kXEpiWarps * 32);
      const uint32_t b = tix & 1, ub = tix >> 1;
      if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      const int t = tt * kGuTok + q * 32 + lane;
      const bool valid = t < T;
      const int sq = valid ? (row_seq ? row_seq[t] : 0) : -1;
      float rs = 0.0f, inv;
      if (sq >= 0) seq_scale_ref(a_absmax[sq], &rs, &inv);
      const float* rg = s_rsc + cur * 2 * kGuCh + half * 64;
      const float* ru = rg + kGuCh;
      const uint32_t tb = t_lane + b * (2 * kGuCh) + half * 64;
      float* dst = h_out + (size_t)(valid ? t : 0) * F + ct * kGuCh + half * 64;
      float run = 0.0f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t g[16], u[16];
        tmem_ld16(tb + c * 16, g);
        tmem_ld16(tb + kGuCh + c * 16, u);
        tmem_wait_ld();
        reg_barrier16(g);
        reg_barrier16(u);
        if (c == 3) {  // every value of this tile is in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
        float hv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hv[i] = gelu_up_f(__fmul_rn(__uint_as_float(g[i]), rg[c * 16 + i]),
                            __fmul_rn(__uint_as_float(u[i]), ru[c * 16 + i]), rs);
          run = fmaxf(run, fabsf(hv[i]));
        }
        if (valid) {
          float4* d4 = reinterpret_cast<float4*>(dst + c * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_float4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
        }
      }
      if (out_absmax) {
        const int s0 = __shfl_sync(0xffffffffu, sq, 0);
        if (__all_sync(0xffffffffu, sq == s0)) {
          const float mx = warp_max(run);
          if (lane == 0 && s0 >= 0) atomicMax(&out_absmax[s0], __float_as_uint(mx));
        } else if (sq >= 0) {
          atomicMax(&out_absmax[sq], __float_as_uint(run));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

namespace {

int g_split_sms[64];
bool g_split_attr[64][2];
std::mutex g_split_mu;

template <int EPI>
cudaError_t launch_split(const __half* a_codes, const __half* w_hi, const __half* w_lo, const float* row_scale, int T,
                         int n_rows, int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c,
                         uint32_t* out_absmax, uint32_t* err, cudaStream_t stream) {
  using Cf = XCfg<EPI>;
  using L = XLayout<EPI>;
  auto kern = gemm_q8_split_kernel<EPI>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int sms;
  {
    std::lock_guard<std::mutex> lk(g_split_mu);
    if (!g_split_sms[dev] &&
        (e = cudaDeviceGetAttribute(&g_split_sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    const int slot = EPI == kEpiStore ? 0 : 1;
    if (!g_split_attr[dev][slot]) {
      if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem)) != cudaSuccess)
        return e;
      g_split_attr[dev][slot] = true;
    }
    sms = g_split_sms[dev];
  }
  const int n_per_a = n_rows / Cf::NA;
  CUtensorMap tm_w, tm_a;
  {  // (K, rows, plane): the lo plane follows the hi plane
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)n_rows, 2};
    const uint64_t strides[2] = {(uint64_t)K * 2, (uint64_t)n_rows * K * 2};
    const uint32_t box[3] = {kXK, kXM, 2};
    if ((e = tmap_nd(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w_hi, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) !=
        cudaSuccess)
      return e;
  }
  if ((e = tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_codes, T, K, kXK, Cf::NT,
                   CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
    return e;
  const int total = (n_per_a / kXM) * ((T + Cf::NT - 1) / Cf::NT);
  const int grid = total < sms ? total : sms;
  kern<<<grid, kXThreads, L::kSmem, stream>>>(tm_w, tm_a, row_scale, n_per_a, T, K, a_absmax, row_seq, c,
                                              out_absmax, err);
  return cudaGetLastError();
}

bool g_gu_attr[64];

cudaError_t launch_gateup(const __half* a_codes, const __half* w_hi, const __half* w_lo, const float* row_scale, int T,
                          int F, int K, const uint32_t* a_absmax, const int32_t* row_seq, float* h, uint32_t* out_absmax,
                          uint32_t* err, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int sms;
  {
    std::lock_guard<std::mutex> lk(g_split_mu);
    if (!g_split_sms[dev] &&
        (e = cudaDeviceGetAttribute(&g_split_sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    if (!g_gu_attr[dev]) {
      if ((e = cudaFuncSetAttribute(gemm_q8_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGuSmem)) !=
          cudaSuccess)
        return e;
      g_gu_attr[dev] = true;
    }
    sms = g_split_sms[dev];
  }
  CUtensorMap tm_w, tm_a;
  {  // (K, channel, gate/up, plane): up rows F below gate rows, the lo plane after the hi plane
    const uint64_t dims[4] = {(uint64_t)K, (uint64_t)F, 2, 2};
    const uint64_t strides[3] = {(uint64_t)K * 2, (uint64_t)F * K * 2, (uint64_t)2 * F * K * 2};
    const uint32_t box[4] = {kXK, kGuCh, 2, 2};
    if ((e = tmap_nd(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w_hi, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) !=
        cudaSuccess)
      return e;
  }
  if ((e = tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_codes, T, K, kXK, kGuTok,
                   CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
    return e;
  const int total = (F / kGuCh) * ((T + kGuTok - 1) / kGuTok);
  const int grid = total < sms ? total : sms;
  gemm_q8_gateup_kernel<<<grid, kXThreads, kGuSmem, stream>>>(tm_w, tm_a, row_scale, F, T, K, a_absmax, row_seq,
                                                              h, out_absmax, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_q8_split(const __half* a_codes, const __half* w_hi, const __half* w_lo, const float* row_scale,
                                 int M, int N, int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c,
                                 int epilogue, uint32_t* out_absmax, uint32_t* err, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (M < 0 || K <= 0 || K % kXK != 0) return cudaErrorInvalidValue;
  if (w_lo != w_hi + (size_t)N * K) return cudaErrorInvalidValue;  // one map covers both planes
  if (epilogue == kEpiGeluUp) {
    if (N % (2 * kGuCh) != 0) return cudaErrorInvalidValue;
    return launch_gateup(a_codes, w_hi, w_lo, row_scale, M, N / 2, K, a_absmax, row_seq, c, out_absmax, err, stream);
  }
  if (N % kXM != 0) return cudaErrorInvalidValue;
  return launch_split<kEpiStore>(a_codes, w_hi, w_lo, row_scale, M, N, K, a_absmax, row_seq, c, nullptr, err, stream);
}

namespace {
std::atomic<int> g_q8_path{0};  // 0 auto, 1 per-block, 2 split (long rows), 3 split (all rows)
}  // namespace

int set_q8_path(int mode) {
  if (mode < 0 || mode > 3) return -1;
  return g_q8_path.exchange(mode);
}

int get_q8_path() { return g_q8_path.load(std::memory_order_relaxed); }

cudaError_t launch_q8_proj(const __half* a_codes, const Q8Proj& w, int M, int N, int K, const uint32_t* a_absmax,
                           const int32_t* row_seq, float* c, int epilogue, uint32_t* out_absmax, uint32_t* err,
                           cudaStream_t stream) {
  const int path = g_q8_path.load(std::memory_order_relaxed);
  if (path != 1 && w.hi && w.lo && w.row_scale && K % kXK == 0) {
    if (path >= 2)
      return launch_gemm_q8_split(a_codes, w.hi, w.lo, w.row_scale, M, N, K, a_absmax, row_seq, c, epilogue,
                                  out_absmax, err, stream);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
      std::lock_guard<std::mutex> lk(g_split_mu);
      if (!g_split_sms[dev]) cudaDeviceGetAttribute(&g_split_sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (g_split_sms[dev] > 0) sms = g_split_sms[dev];
    }
    const bool gelu = epilogue == kEpiGeluUp;
    const int nt = gelu ? kGuTok : XCfg<kEpiStore>::NT;
    const int64_t tiles = (int64_t)(N / (gelu ? 2 : 1) / kXM) * ((M + nt - 1) / nt);
    if (2 * tiles >= sms)  // measured crossover: from ~half a wave of split tiles it beats the per-block kernel
      return launch_gemm_q8_split(a_codes, w.hi, w.lo, w.row_scale, M, N, K, a_absmax, row_seq, c, epilogue,
                                  out_absmax, err, stream);
  }
  return launch_gemm_q8(a_codes, w.codes, w.scales, M, N, K, a_absmax, row_seq, c, epilogue, out_absmax, err, stream);
}

}  // namespace sem
