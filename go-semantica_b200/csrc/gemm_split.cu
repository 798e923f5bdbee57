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
// QKV, O and down (gemm_q8_pair_kernel) run on SM pairs: clusters of two
// CTAs whose leader issues cta_group::2 MMAs of M = 256 weight rows (128 per
// CTA) by N = 256 tokens (128 staged per CTA), so each SM stages 48 KB per
// 1024 MMA cycles where a single-SM tile needs 64 KB. Gate/up
// (gemm_q8_gateup_kernel) stays on one SM: tokens are M = 128, the gate and
// up rows of 128 channels together are N = 256, and its GELU epilogue, not
// operand traffic, sets its pace (a pair version measured slower). Both keep
// two tiles' accumulators in TMEM (512 columns) so the epilogue of tile i
// overlaps the MMAs of tile i+1, with one persistent CTA per SM: warps 0 and 2
// issue TMA for alternate stages, warp 1 (of the pair leader) the MMAs, and
// two (store) or four (gate/up) warps per TMEM lane quarter the epilogue.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.h"

namespace sem {

namespace {

constexpr int kXK = 64;                    // K elements per stage: 128 bytes of fp16 per row
constexpr int kXRows = 128;                // rows of each operand half per CTA (TMEM lanes)
constexpr int kXTile = kXRows * kXK * 2;   // 16 KB: 128 rows x 128 bytes
constexpr int kXStage = 3 * kXTile;        // 48 KB per CTA and stage: two weight planes and one token tile
constexpr int kXStages = 4;
constexpr int kXEpiWarps = 8;                       // two per TMEM lane quarter
constexpr int kXThreads = 128 + 32 * kXEpiWarps;    // warps 0-3: TMA, MMA, TMA, idle
constexpr int kXBarBytes = 256;
constexpr int kXPairTok = 2 * kXRows;      // tokens per pair tile
constexpr int kXSmem = 1024 + kXStages * kXStage + kXBarBytes + 2 * kXPairTok * 4;
static_assert(kXSmem <= 232448, "shared memory per CTA");
static_assert((2 * kXStages + 5) * 8 + 8 <= kXBarBytes, "barrier block");
constexpr uint16_t kPairMask = 0x3;        // both CTAs of the pair

__device__ uint32_t g_split_error;  // error bits of launches given no error word

// GELUQuick(gate * rs) * (up * rs), the runMLPINT8 element (model_int8.go:523-530).
// Scalar on purpose: ptxas contracts a packed (f32x2) multiply with the add
// that consumes it into one fused multiply-add even when both carry .rn, which
// would change fastExp's polynomial in the last bit.
__device__ __forceinline__ float gelu_up_f(float g, float u, float rs) {
  return __fmul_rn(gelu_quick_ref(__fmul_rn(g, rs)), __fmul_rn(u, rs));
}

}  // namespace

// QKV, O and down on SM pairs (clusters of two CTAs, one per SM). Per stage
// each CTA stages 128 weight rows x 64 K of the hi and lo planes (A: rows
// [256 mt + 128 rank, +128)) and 128 of the tile's 256 tokens (B); the
// leader's M = 256, N = 256 MMAs read both CTAs' tiles, so each SM moves 48 KB
// per 1024 MMA cycles instead of the 64 KB of a single-SM tile. Each CTA's
// accumulator is its 128 output channels x the 256 tokens.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kXThreads, 1)
    gemm_q8_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                        const float* __restrict__ row_scale, int n_out, int T, int K,
                        const uint32_t* __restrict__ a_absmax, const int32_t* __restrict__ row_seq,
                        float* __restrict__ c_out, uint32_t* __restrict__ err, VPlanes vp) {
  constexpr int ST = kXStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * kXStage);  // leader: both CTAs' bytes
  uint64_t* empty = full + ST;                                         // each CTA: stage consumed
  uint64_t* tfull = empty + ST;                                        // each CTA: accumulator ready
  uint64_t* tempty = tfull + 2;                                        // leader: both epilogues done
  uint64_t* drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_sc = reinterpret_cast<float*>(smem + ST * kXStage + kXBarBytes);  // [2][256] epilogue scales
  if (!err) err = &g_split_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // output tiles: (256-token tile, 256-row weight tile); a 128-row tail leaves the peer's half empty
  const int n_wt = (n_out + 2 * kXRows - 1) / (2 * kXRows);
  const int total = n_wt * ((T + kXPairTok - 1) / kXPairTok);
  const int nks = K / kXK;

  if (threadIdx.x == 0) {
    for (int st = 0; st < ST; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kXEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers (alternate stages), both CTAs ----------------
    if (lane == 0) {
      const uint32_t me = warp >> 1;
      const uint32_t lead_full = mapa_shared(smem_u32(full), 0);
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_a);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total; tile += npairs) {
        const int tt = tile / n_wt, wt = tile % n_wt;
        const int tok = tt * kXPairTok + (int)rank * kXRows;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          if ((it & 1) != me) continue;
          const uint32_t st = it % ST, u = it / ST;
          if (!mbar_wait(&empty[st], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          uint8_t* sp = stages + st * kXStage;
          const uint32_t cbar = lead_full + 8 * st;
          if (rank == 0) mbar_arrive_expect_tx(&full[st], 2 * kXStage);
          // [hi, lo][128 rows][128 B]: one 3-D copy, then the tokens
          tma_load_3d_pair(&tm_w, cbar, sp, ks * kXK, (2 * wt + (int)rank) * kXRows, 0);
          tma_load_2d_pair(&tm_a, cbar, sp + 2 * kXTile, ks * kXK, tok);
        }
      }
      // The leader's full barriers count both CTAs' bytes: copies in flight
      // land before either CTA's shared memory is released.
      if (rank == 0)
        for (uint32_t j = it > (uint32_t)ST ? it - ST : 0; j < it; ++j)
          if ((j & 1) == me) mbar_wait_drain(&full[j % ST], (j / ST) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the leader's thread drives both SMs ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(2 * kXRows, 2 * kXRows);
      uint32_t it = 0, tix = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total; tile += npairs, ++tix) {
        const uint32_t b = tix & 1, ub = tix >> 1;
        if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + b * 256;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const uint32_t st = it % ST, u = it / ST;
          if (!mbar_wait(&full[st], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sp = smem_u32(stages + st * kXStage);
#pragma unroll
          for (int kk = 0; kk < kXK / 16; ++kk) {
            const uint64_t bdesc = umma_desc_k_sw128(sp + 2 * kXTile + kk * 32);
            umma_f16_pair(d0, umma_desc_k_sw128(sp + kk * 32), bdesc, idesc, (ks | kk) ? 1u : 0u);
            umma_f16_pair(d0, umma_desc_k_sw128(sp + kXTile + kk * 32), bdesc, idesc, 1u);
          }
          umma_commit_pair_mc(&empty[st], kPairMask);
        }
        if (!ok) break;
        umma_commit_pair_mc(&tfull[b], kPairMask);
      }
      umma_commit_pair_mc(drain, 0x1);  // every MMA has finished writing TMEM before it is freed
      mbar_wait_drain(drain, 0);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue, both CTAs: this CTA's 128 TMEM lanes ----------------
    const int e = warp - 4;
    const int q = warp & 3;    // the TMEM lane quarter this warp may access
    const int half = e >> 2;   // half of the tile's 256 tokens
    const int etid = e * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t lead_tempty = mapa_shared(smem_u32(tempty), 0);
    bool ok = true;
    uint32_t tix = 0;
    for (int tile = pair; tile < total; tile += npairs, ++tix) {
      const int tt = tile / n_wt, wt = tile % n_wt;
      const int cur = tix & 1;
      float* sc = s_sc + cur * kXPairTok;
      {  // the input scale of each of the tile's 256 tokens (double-buffered across tiles)
        const int t = tt * kXPairTok + etid;
        const int sq = t < T ? (row_seq ? row_seq[t] : 0) : -1;
        float rs = 0.0f, inv;
        if (sq >= 0) seq_scale_ref(a_absmax[sq], &rs, &inv);
        sc[etid] = rs;
      }
      named_bar_sync(1, kXEpiWarps * 32);
      const uint32_t b = tix & 1, ub = tix >> 1;
      if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);  // converged (and agreed) before the .sync.aligned TMEM loads
      if (!ok) continue;
      tc_fence_after();
      constexpr int TPH = kXPairTok / 2;  // tokens of a thread's half of the tile
      const int n0 = (2 * wt + (int)rank) * kXRows + q * 32 + lane;  // output channel
      const bool live = (2 * wt + (int)rank) * kXRows < n_out;      // uniform: a 128-row tail half is empty
      const uint32_t tb = t_lane + b * 256 + half * TPH;
      const float* c_rs = sc + half * TPH;
      const int tok0 = tt * kXPairTok + half * TPH;  // first token of this thread's half
      const float rsc = live ? row_scale[n0] : 0.0f;
      float* dst = c_out + (size_t)tok0 * n_out + n0;
      // a tile of V columns (uniform: the V block starts on a 128-row tile)
      // goes to the attention's fp16 hi / lo planes instead
      const bool vtile = vp.hi && (2 * wt + (int)rank) * kXRows >= vp.col0;
      __half* vhp = vtile ? vp.hi + (size_t)tok0 * 256 + (n0 - vp.col0) : nullptr;
      __half* vlp = vtile ? vhp + (size_t)vp.rows * 256 : nullptr;
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
          if (lane == 0) mbar_arrive_cluster(lead_tempty + 8 * b);
        }
        if (!live) continue;
        float crs[2][16];  // the tokens' input scales, four 16-byte loads per 16 tokens
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<float4*>(crs[cc])[i] = reinterpret_cast<const float4*>(c_rs + (c + cc) * 16)[i];
        if (!vtile) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int x = (c + cc) * 16 + i;
              if (tok0 + x < T)  // warp-uniform
                dst[(size_t)x * n_out] = __fmul_rn(__fmul_rn(__uint_as_float(r[cc][i]), rsc), crs[cc][i]);
            }
        } else {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int x = (c + cc) * 16 + i;
              if (tok0 + x < T) {  // warp-uniform
                const float v = __fmul_rn(__fmul_rn(__uint_as_float(r[cc][i]), rsc), crs[cc][i]);
                __half hi, lo;
                split_half(v, hi, lo);
                vhp[(size_t)x * 256] = hi;
                vlp[(size_t)x * 256] = lo;
              }
            }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs have drained; no copy or arrival is still aimed at either CTA
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
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
constexpr int kGuEpiWarps = 16;  // four per TMEM lane quarter: the GELU epilogue costs about as much as the MMAs
constexpr int kGuThreads = 128 + 32 * kGuEpiWarps;
static_assert(kGuSmem <= 232448, "shared memory per CTA");

__global__ void __launch_bounds__(kGuThreads, 1)
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
      mbar_init(&tempty[b], kGuEpiWarps);
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
    const int part = e >> 2;    // channels [32 part, +32) of the tile
    const int etid = e * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    uint32_t tix = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tix) {
      const int tt = tile / n_ct, ct = tile % n_ct;
      const int cur = tix & 1;
      // the channels' row scales of this tile (double-buffered across tiles)
      if (etid < 2 * kGuCh)
        s_rsc[cur * 2 * kGuCh + etid] =
            row_scale[(etid < kGuCh ? 0 : F - kGuCh) + ct * kGuCh + etid];  // gate rows, then up rows
      named_bar_sync(1, kGuEpiWarps * 32);
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
      const float* rg = s_rsc + cur * 2 * kGuCh + part * 32;
      const float* ru = rg + kGuCh;
      const uint32_t tb = t_lane + b * (2 * kGuCh) + part * 32;
      float* dst = h_out + (size_t)(valid ? t : 0) * F + ct * kGuCh + part * 32;
      float run = 0.0f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t g[16], u[16];
        tmem_ld16(tb + c * 16, g);
        tmem_ld16(tb + kGuCh + c * 16, u);
        tmem_wait_ld();
        reg_barrier16(g);
        reg_barrier16(u);
        if (c == 1) {  // every value of this tile is in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
        float hv[16], sg[16], su[16];  // the channels' row scales, four 16-byte loads each
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          reinterpret_cast<float4*>(sg)[i] = reinterpret_cast<const float4*>(rg + c * 16)[i];
          reinterpret_cast<float4*>(su)[i] = reinterpret_cast<const float4*>(ru + c * 16)[i];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hv[i] = gelu_up_f(__fmul_rn(__uint_as_float(g[i]), sg[i]), __fmul_rn(__uint_as_float(u[i]), su[i]), rs);
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
bool g_split_attr[64];
std::mutex g_split_mu;

cudaError_t launch_pair(const __half* a_codes, const __half* w_hi, const float* row_scale, int T, int n_out, int K,
                        const uint32_t* a_absmax, const int32_t* row_seq, float* c, uint32_t* err, cudaStream_t stream,
                        const VPlanes& vp) {
  if (vp.hi && (vp.col0 % kXRows != 0 || n_out - vp.col0 != 256 || vp.rows < T)) return cudaErrorInvalidValue;
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
    if (!g_split_attr[dev]) {
      if ((e = cudaFuncSetAttribute(gemm_q8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kXSmem)) !=
          cudaSuccess)
        return e;
      g_split_attr[dev] = true;
    }
    sms = g_split_sms[dev];
  }
  CUtensorMap tm_w, tm_a;
  {  // (K, rows, plane): the lo plane follows the hi plane
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)n_out, 2};
    const uint64_t strides[2] = {(uint64_t)K * 2, (uint64_t)n_out * K * 2};
    const uint32_t box[3] = {kXK, kXRows, 2};
    if ((e = tmap_nd(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w_hi, 3, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
      return e;
  }
  if ((e = tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_codes, T, K, kXK, kXRows,
                   CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
    return e;
  const int n_wt = (n_out + 2 * kXRows - 1) / (2 * kXRows);
  const int total = n_wt * ((T + kXPairTok - 1) / kXPairTok);
  const int pairs = total < sms / 2 ? total : sms / 2;
  gemm_q8_pair_kernel<<<2 * pairs, kXThreads, kXSmem, stream>>>(tm_w, tm_a, row_scale, n_out, T, K, a_absmax,
                                                                row_seq, c, err, vp);
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
  gemm_q8_gateup_kernel<<<grid, kGuThreads, kGuSmem, stream>>>(tm_w, tm_a, row_scale, F, T, K, a_absmax, row_seq,
                                                              h, out_absmax, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_q8_split(const __half* a_codes, const __half* w_hi, const __half* w_lo, const float* row_scale,
                                 int M, int N, int K, const uint32_t* a_absmax, const int32_t* row_seq, float* c,
                                 int epilogue, uint32_t* out_absmax, uint32_t* err, cudaStream_t stream,
                                 const VPlanes& vp) {
  if (M == 0) return cudaSuccess;
  if (M < 0 || K <= 0 || K % kXK != 0) return cudaErrorInvalidValue;
  if (w_lo != w_hi + (size_t)N * K) return cudaErrorInvalidValue;  // one map covers both planes
  if (epilogue == kEpiGeluUp) {
    if (N % (2 * kXRows) != 0) return cudaErrorInvalidValue;
    return launch_gateup(a_codes, w_hi, w_hi + (size_t)N * K, row_scale, M, N / 2, K, a_absmax, row_seq, c, out_absmax,
                         err, stream);
  }
  if (N % kXRows != 0) return cudaErrorInvalidValue;
  return launch_pair(a_codes, w_hi, row_scale, M, N, K, a_absmax, row_seq, c, err, stream, vp);
}

namespace {
// 0 auto, 1 per-block, 2 split (long rows), 3 split (all rows), 4 CUDA-core VNNI order (all rows)
std::atomic<int> g_q8_path{0};
}  // namespace

int set_q8_path(int mode) {
  if (mode < 0 || mode > 4) return -1;
  return g_q8_path.exchange(mode);
}

int get_q8_path() { return g_q8_path.load(std::memory_order_relaxed); }

namespace {
enum Q8Kernel { kQ8Dp4a, kQ8Split, kQ8Block };

// The kernel launch_q8_proj takes for these operands (see kernels.h).
Q8Kernel q8_choice(const Q8Proj& w, int M, int N, int K, int epilogue) {
  const int path = g_q8_path.load(std::memory_order_relaxed);
  // Below 128 rows (and everywhere under path 4) the CUDA-core kernel: the
  // reference's VNNI float32 order exactly, and no tensor-core pipeline to
  // fill for a handful of tiles.
  if (w.lanes && (path == 4 || (path == 0 && M < kDp4aMaxRows))) return kQ8Dp4a;
  if (path != 1 && w.hi && w.lo && w.row_scale && K % kXK == 0) {
    if (path >= 2) return kQ8Split;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
      std::lock_guard<std::mutex> lk(g_split_mu);
      if (!g_split_sms[dev]) cudaDeviceGetAttribute(&g_split_sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (g_split_sms[dev] > 0) sms = g_split_sms[dev];
    }
    // 128-row x 256-token units (a pair tile is two): the measured crossover
    // is about half a wave of them
    const int64_t tiles = (int64_t)(N / (epilogue == kEpiGeluUp ? 2 : 1) / kXRows) * ((M + 255) / 256);
    if (2 * tiles >= sms) return kQ8Split;
  }
  return kQ8Block;
}
}  // namespace

cudaError_t launch_q8_proj(const __half* a_codes, const Q8Proj& w, int M, int N, int K, const uint32_t* a_absmax,
                           const int32_t* row_seq, float* c, int epilogue, uint32_t* out_absmax, uint32_t* err,
                           cudaStream_t stream, const VPlanes& vp) {
  const Q8Kernel kern = q8_choice(w, M, N, K, epilogue);
  const bool v = vp.hi && M > 0 && epilogue == kEpiStore && kern == kQ8Split;
  if (vp.written) *vp.written = v;
  switch (kern) {
    case kQ8Dp4a:
      return launch_gemm_q8_dp4a(a_codes, w.lanes, w.scales, M, N, K, a_absmax, row_seq, c, epilogue, out_absmax,
                                 stream);
    case kQ8Split:
      return launch_gemm_q8_split(a_codes, w.hi, w.lo, w.row_scale, M, N, K, a_absmax, row_seq, c, epilogue,
                                  out_absmax, err, stream, v ? vp : VPlanes{});
    default:
      return launch_gemm_q8(a_codes, w.codes, w.scales, M, N, K, a_absmax, row_seq, c, epilogue, out_absmax, err,
                            stream);
  }
}

}  // namespace sem
