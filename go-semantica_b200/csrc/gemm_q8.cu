// Q8_0 weights x INT8 activations (MatMulQ8_0INT8, internal/kernels/quantize.go:346-458)
// on the sm_100a tensor cores (tcgen05, accumulators in TMEM).
//
// The reference sums the int8 products of each 32-element Q8_0 block exactly
// and only then applies the block's fp16 scale in float32:
//   dst[t, j] = inScale * sum_kb float32(sum_{k in kb} a[t, k] * q[j, k]) * d[j, kb].
// Here both operands hold those integers as fp16 (|a|, |q| <= 127 are exact)
// and one K = 32 block is two kind::f16 MMAs with an fp32 accumulator: the
// products and their sums (|sum| < 2^19) are integers below 2^24, so every
// block sum lands in TMEM exactly. The epilogue warps read each block's sums
// from TMEM and apply the block scale with packed fp32 FMAs into register
// accumulators, blocks in ascending order -- the reference's arithmetic up to
// the float32 order of the block accumulation.
//
// Roles: the weight rows (output channels) are the MMA's M = 128 (TMEM lanes),
// so each epilogue thread owns one channel and its block scale is a scalar;
// the tokens are N. Warps 0 and 2 issue TMA loads for alternate stages
// (128-byte swizzled K-major tiles, 4-stage ring of 64-wide K slices), warp 1
// issues the MMAs, warps 4-15 drain
// TMEM: three groups of four warps (one per TMEM lane quarter), each group a
// third of the tile's tokens, so a thread accumulates 64 values and every
// block costs it one batch of TMEM loads and one wait. TMEM holds two block
// buffers: the MMA of block kb+1 overlaps the epilogue of block kb.
// Results leave through shared-memory staging and asynchronous TMA stores of
// 16-token boxes, so the next tile's MMAs are not held up by the stores.
// The gate/up projection (runMLPINT8, model_int8.go:510-538) runs both weight
// matrices against the same token tile into two TMEM regions; its epilogue
// forms GELUQuick(gate) * up in shared memory and the per-sequence absmax.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sem {

namespace {

constexpr int kBM = 128;       // weight rows per tile (TMEM lanes)
constexpr int kBKS = 64;       // K elements per pipeline stage: two Q8_0 blocks, 128 bytes of fp16
constexpr int kStages = 4;
static_assert(kStages % 2 == 0, "the two TMA threads own alternate stages");
constexpr int kATile = kBM * kBKS * 2;      // 16 KB
constexpr int kSubTok = 16;                 // tokens per output box
constexpr int kOutBox = kSubTok * kBM * 4;  // 8 KB: one fp32 box of 16 tokens x 128 channels
constexpr int kBarBytes = 160;              // up to 21 mbarriers + TMEM address + abort flag, 16-byte padded
constexpr int kRegsProducer = 56;           // warpgroup 0 after setmaxnreg.dec

// NA weight operands x NT tokens per tile; GR token groups of four epilogue
// warps (one per TMEM lane quarter). Warpgroup 0: TMA warps 0 and 2, MMA warp
// 1, idle warp 3; then GR epilogue warpgroups. TMEM holds kNB block buffers
// (up to four), so the MMAs may run that many blocks ahead of the epilogue.
template <int NA, int NT, int GR>
struct TileCfg {
  static constexpr int kEpiWarps = 4 * GR;
  static constexpr int kEpiThreads = kEpiWarps * 32;
  static constexpr int kThreads = 128 + kEpiThreads;
  // register split (setmaxnreg): the launch gets 65536 / kThreads per thread
  // (rounded down to a multiple of 8); warpgroup 0 gives up all but 56
  static constexpr int kRegsLaunch = (65536 / kThreads) / 8 * 8 > 255 ? 248 : (65536 / kThreads) / 8 * 8;
  static constexpr int kRegsEpilogue = GR >= 3 ? 152 : 192;
  static_assert(128 * kRegsProducer + kEpiThreads * kRegsEpilogue <= kThreads * kRegsLaunch, "register split");
  static constexpr int kTG = NT / GR;         // tokens per epilogue group
  static constexpr int kCPO = kTG / 16;       // TMEM chunks of 16 columns per operand
  static constexpr int kChunks = NA * kCPO;
  static constexpr int kPairs = kChunks * 8;  // packed fp32 pairs accumulated per thread
  static constexpr int kBTile = NT * kBKS * 2;
  static constexpr int kStage = NA * kATile + kBTile;  // bytes per stage (also the TMA transaction count)
  static constexpr int kBufCols = NA * NT;             // TMEM columns of one block buffer
  static constexpr int kNB = 512 / kBufCols >= 4 ? 4 : 512 / kBufCols;
  static constexpr int kTmemCols = kNB * kBufCols <= 256 ? 256 : 512;
  static constexpr int kOutBytes = GR * 2 * kOutBox;  // per group: two boxes (double buffer, or gate + up)
  static constexpr int kSmem = 1024 + kStages * kStage + kOutBytes + kBarBytes + NT * 16;
  static_assert(NT % (16 * GR) == 0 && kTG % kSubTok == 0, "token tile must split into 16-token boxes");
  static_assert(kNB >= 2, "at least two block buffers in TMEM");
  static_assert(2 * kStages + 2 * kNB + 1 <= (kBarBytes - 8) / 8, "barrier block");
  static_assert(kChunks <= 4, "register budget: at most 64 accumulators and 64 staging registers per thread");
  static_assert(kSmem <= 232448, "shared memory per CTA");
};

__device__ uint32_t g_tc_error;  // error bits of launches given no error word

// TMEM column of chunk c (16 columns) of a group's share of a block buffer:
// operand c / kCPO, then the group's third of the tokens.
template <int NA, int NT, int GR>
__device__ __forceinline__ uint32_t chunk_col(int grp, int c) {
  constexpr int cpo = TileCfg<NA, NT, GR>::kCPO;
  return (uint32_t)((c / cpo) * NT + grp * TileCfg<NA, NT, GR>::kTG + (c % cpo) * 16);
}

__device__ __forceinline__ float f4_get(const float4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  // Ties the loaded registers to the wait so that no use is scheduled before it.
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// GELUQuick(gate * rs) * (up * rs); called from a rolled loop, so one copy.
__device__ __forceinline__ float gelu_up(float g, float u, float rs) {
  return __fmul_rn(gelu_quick_ref(__fmul_rn(g, rs)), __fmul_rn(u, rs));
}

}  // namespace

// One persistent CTA per SM walks tiles (128 weight rows x NT tokens), tile
// index = token tile * n_mt + weight tile, so the CTAs working at one time
// share a few token tiles through L2.
template <int NA, int NT, int GR, int EPI>
__global__ void __launch_bounds__(TileCfg<NA, NT, GR>::kThreads, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_c, const float* __restrict__ ws, int w_rows,
                      int n_per_a, int T, int K, const uint32_t* __restrict__ a_absmax,
                      const int32_t* __restrict__ row_seq, uint32_t* __restrict__ out_absmax,
                      uint32_t* __restrict__ err, float* __restrict__ Cout) {
  using G = TileCfg<NA, NT, GR>;
  constexpr int NB = G::kNB;
  constexpr int kEpiWarps = G::kEpiWarps, kEpiThreads = G::kEpiThreads;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* stages = smem;
  uint8_t* outbuf = smem + kStages * G::kStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(outbuf + G::kOutBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + NB;
  uint64_t* drain = tempty + NB;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_rs = reinterpret_cast<float*>(outbuf + G::kOutBytes + kBarBytes);
  int* s_seq = reinterpret_cast<int*>(s_rs + 2 * NT);
  if (!err) err = &g_tc_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mt = n_per_a / kBM;
  const int total = n_mt * ((T + NT - 1) / NT);
  const int nks = K / kBKS, nkb = K / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, G::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers ----------------
    // Two threads (warps 0 and 2) issue alternate stages: the tile loads of
    // one thread complete at a limited rate (a few copies in flight), so a
    // second stream doubles the L2 -> SM rate of the SM.
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
          const uint32_t s = it % kStages, u = it / kStages;
          if (!mbar_wait(&empty[s], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + s * G::kStage;
          mbar_arrive_expect_tx(&full[s], G::kStage);
#pragma unroll
          for (int a = 0; a < NA; ++a) tma_load_2d(&tm_w, &full[s], st + a * kATile, ks * kBKS, a * n_per_a + mt * kBM);
          tma_load_2d(&tm_a, &full[s], st + NA * kATile, ks * kBKS, tt * NT);
        }
      }
      // the copies in flight land before the CTA's shared memory is released
      // (`it` is one past the last iteration this thread issued or skipped;
      // stage s is only ever used by thread s & 1, kStages being even)
      for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0; j < it; ++j)
        if ((j & 1) == me) mbar_wait_drain(&full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(kBM, NT);
      uint32_t it = 0, blk = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const uint32_t s = it % kStages, u = it / kStages;
          if (!mbar_wait(&full[s], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + s * G::kStage);
          for (int h = 0; h < 2 && ok; ++h, ++blk) {
            const uint32_t b = blk % NB, ub = blk / NB;
            if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int a = 0; a < NA; ++a)
#pragma unroll
              for (int kk = 0; kk < 2; ++kk) {
                const uint32_t koff = (uint32_t)(h * 2 + kk) * 32;
                umma_f16(tmem_base + b * G::kBufCols + a * NT, umma_desc_k_sw128(sa + a * kATile + koff),
                         umma_desc_k_sw128(sa + NA * kATile + koff), idesc, (uint32_t)kk);
              }
            umma_commit(&tfull[b]);
          }
          if (!ok) break;
          umma_commit(&empty[s]);
        }
      }
      umma_commit(drain);  // every MMA has finished writing TMEM before it is freed
      mbar_wait_drain(drain, 0);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(G::kRegsEpilogue));
    // ---------------- epilogue: TMEM -> scaled fp32 accumulators -> output ----------------
    constexpr int CH = G::kChunks, NP = G::kPairs, NPA = NP / NA, TG = G::kTG;
    const int e = warp - 4;
    const int q = warp & 3;      // the TMEM lane quarter this warp may access
    const int grp = e >> 2;      // which third of the tile's tokens
    const int etid = e * 32 + lane;
    const int ch = q * 32 + lane;  // channel within the tile
    const bool leader = (e & 3) == 0 && lane == 0;  // issues the group's TMA stores
    float* gbox = reinterpret_cast<float*>(outbuf + grp * 2 * kOutBox);  // two [16][128] fp32 boxes
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    uint32_t blk = 0;
    int nstore = 0;  // stores issued by this group (double-buffer index)
    bool ok = true;  // after an abort every warp still walks the same named barriers
    // per-token activation scale and sequence of a tile, double-buffered: the
    // next tile's entries are loaded while this tile accumulates
    auto tile_token = [&](int tile_idx) { return (tile_idx / n_mt) * NT + etid; };
    auto seq_of = [&](int t) { return t < T ? (row_seq ? row_seq[t] : 0) : -1; };
    if (etid < NT && (int)blockIdx.x < total) {
      const int sq = seq_of(tile_token(blockIdx.x));
      float rs = 0.0f, inv;
      if (sq >= 0) seq_scale_ref(a_absmax[sq], &rs, &inv);
      s_rs[etid] = rs;
      s_seq[etid] = sq;
    }
    // block scales of this thread's weight row(s), row-major [row][K/32]: one
    // 16-byte load covers four blocks and is issued a group of four ahead
    auto scale_rows = [&](int mt_, int a) {
      return reinterpret_cast<const float4*>(ws + (size_t)(a * n_per_a + mt_ * kBM + ch) * nkb);
    };
    float4 sa_nxt = make_float4(0.f, 0.f, 0.f, 0.f), sb_nxt = sa_nxt;
    int tix = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tix) {
      const int tt = tile / n_mt, mt = tile % n_mt;
      const int t0 = tt * NT;
      const int cur = tix & 1;
      // this tile's scales are complete; the previous tile's output is done with the other buffer
      named_bar_sync(1, kEpiThreads);
      const float* c_rs = s_rs + cur * NT;
      const int* c_seq = s_seq + cur * NT;
      const int nxt_tile = tile + gridDim.x;
      int nsq = -1;
      uint32_t nrs_bits = 0;
      if (etid < NT && nxt_tile < total) nsq = seq_of(tile_token(nxt_tile));

      uint64_t acc[NP];
#pragma unroll
      for (int i = 0; i < NP; ++i) acc[i] = 0;
      const float4* wsa = scale_rows(mt, 0);
      const float4* wsb = scale_rows(mt, 1);
      if (tix == 0) {
        sa_nxt = wsa[0];
        if (NA == 2) sb_nxt = wsb[0];
      }
      for (int kg = 0; kg < nkb / 4; ++kg) {
        const float4 sa_cur = sa_nxt, sb_cur = sb_nxt;
        if (kg + 1 < nkb / 4) {
          sa_nxt = wsa[kg + 1];
          if (NA == 2) sb_nxt = wsb[kg + 1];
        } else if (nxt_tile < total) {  // the next tile's first group
          sa_nxt = scale_rows(nxt_tile % n_mt, 0)[0];
          if (NA == 2) sb_nxt = scale_rows(nxt_tile % n_mt, 1)[0];
        }
        if (kg == 1) {  // the next tile's activation scales: second, dependent load
          nrs_bits = nsq >= 0 ? a_absmax[nsq] : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u, ++blk) {
        const uint32_t b = blk % NB, ub = blk / NB;
        if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
        ok = __all_sync(0xffffffffu, ok);  // converged (and agreed) before the .sync.aligned TMEM loads
        if (ok) {
          tc_fence_after();
          const uint32_t tb = t_lane + b * G::kBufCols;
          const float da = f4_get(sa_cur, u), db = f4_get(sb_cur, u);
          const uint64_t dd0 = pack2(da, da), dd1 = pack2(db, db);
          // two chunks per TMEM wait; the buffer goes back to the MMA after the last wait
#pragma unroll
          for (int hh = 0; hh < CH / 2; ++hh) {
            uint32_t r[2][16];
            tmem_ld16(tb + chunk_col<NA, NT, GR>(grp, 2 * hh), r[0]);
            tmem_ld16(tb + chunk_col<NA, NT, GR>(grp, 2 * hh + 1), r[1]);
            tmem_wait_ld_regs(r[0]);
            reg_barrier16(r[1]);
            if (hh == CH / 2 - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tempty[b]);
            }
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int c = 2 * hh + cc;
              const uint64_t dd = (c / G::kCPO) ? dd1 : dd0;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                acc[c * 8 + i] = fma2(pack2u(r[cc][2 * i], r[cc][2 * i + 1]), dd, acc[c * 8 + i]);
            }
          }
        }
        }
      }

      if (etid < NT && nxt_tile < total) {
        float rs = 0.0f, inv;
        if (nsq >= 0) {
          if (nkb < 8) nrs_bits = a_absmax[nsq];  // no second group: the dependent load was not issued
          seq_scale_ref(nrs_bits, &rs, &inv);
        }
        s_rs[(cur ^ 1) * NT + etid] = rs;
        s_seq[(cur ^ 1) * NT + etid] = nsq;
      }

      // ---- output ----
      const int tg0 = grp * TG;  // first token of this group within the tile
      if (EPI == kEpiStore) {
        // 16-token boxes through shared memory and TMA stores
#pragma unroll
        for (int sbx = 0; sbx < TG / kSubTok; ++sbx) {
          float* out = gbox + (nstore & 1) * (kSubTok * kBM);
          if (leader) bulk_wait_read<1>();  // the store that last read this box is done reading
          named_bar_sync(2 + grp, 128);
          // dst = sum * inputScale (quantize.go:453)
#pragma unroll
          for (int p = 0; p < kSubTok / 2; ++p) {
            float v0, v1;
            unpack2(acc[sbx * (kSubTok / 2) + p], v0, v1);
            const int i = tg0 + sbx * kSubTok + 2 * p;
            out[(2 * p) * kBM + ch] = __fmul_rn(v0, c_rs[i]);
            out[(2 * p + 1) * kBM + ch] = __fmul_rn(v1, c_rs[i + 1]);
          }
          fence_proxy_async_smem();
          named_bar_sync(2 + grp, 128);
          if (leader) {
            tma_store_2d(&tm_c, out, mt * kBM, t0 + tg0 + sbx * kSubTok);
            bulk_commit();
          }
          ++nstore;
        }
      } else {
        // runMLPINT8 (model_int8.go:523-530): gate and up scaled, GELUQuick(gate) * up,
        // and the absmax of each sequence's rows for the next quantisation. Gate
        // and up of 16 tokens go through this thread's own column of two
        // shared-memory boxes (no other thread touches it), so the GELU loop can
        // stay short; h leaves with plain coalesced stores (one 128-byte row of
        // channels per warp and token).
        float* gb = gbox;
        float* ub = gbox + kSubTok * kBM;
        const int j = mt * kBM + ch;
        int cur = -1;
        float run = 0.0f;
#pragma unroll
        for (int sbx = 0; sbx < TG / kSubTok; ++sbx) {
#pragma unroll
          for (int p = 0; p < kSubTok / 2; ++p) {
            float g0, g1, u0, u1;
            unpack2(acc[sbx * (kSubTok / 2) + p], g0, g1);
            unpack2(acc[NPA + sbx * (kSubTok / 2) + p], u0, u1);
            gb[(2 * p) * kBM + ch] = g0;
            gb[(2 * p + 1) * kBM + ch] = g1;
            ub[(2 * p) * kBM + ch] = u0;
            ub[(2 * p + 1) * kBM + ch] = u1;
          }
          const int i0 = tg0 + sbx * kSubTok;
          const int sq0 = c_seq[i0];  // the same for every lane: warp-uniform branches
          if (sq0 >= 0 && sq0 == c_seq[i0 + kSubTok - 1]) {
            // the usual case, 16 tokens of one sequence: no reduction inside the loop,
            // so the unrolled iterations overlap
            if (sq0 != cur) {
              if (cur >= 0 && out_absmax) {
                const float m = warp_max(run);
                if (lane == 0) atomicMax(&out_absmax[cur], __float_as_uint(m));
              }
              cur = sq0;
              run = 0.0f;
            }
            const float rs = c_rs[i0];  // one sequence, one activation scale
            float* dst = Cout + (size_t)(t0 + i0) * n_per_a + j;
#pragma unroll 8
            for (int x = 0; x < kSubTok; ++x) {
              const float h = gelu_up(gb[x * kBM + ch], ub[x * kBM + ch], rs);
              dst[(size_t)x * n_per_a] = h;
              run = fmaxf(run, fabsf(h));
            }
          } else {
#pragma unroll 1
            for (int x = 0; x < kSubTok; ++x) {
              const int i = i0 + x;
              const int sq = c_seq[i];
              if (sq != cur) {
                if (cur >= 0 && out_absmax) {
                  const float m = warp_max(run);
                  if (lane == 0) atomicMax(&out_absmax[cur], __float_as_uint(m));
                }
                cur = sq;
                run = 0.0f;
              }
              if (sq >= 0) {
                const float h = gelu_up(gb[x * kBM + ch], ub[x * kBM + ch], c_rs[i]);
                Cout[(size_t)(t0 + i) * n_per_a + j] = h;
                run = fmaxf(run, fabsf(h));
              }
            }
          }
        }
        if (cur >= 0 && out_absmax) {
          const float m = warp_max(run);
          if (lane == 0) atomicMax(&out_absmax[cur], __float_as_uint(m));
        }
      }
    }
    if (leader) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, G::kTmemCols);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major [rows][cols] 2-D map with a box of box_cols x box_rows.
cudaError_t encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int esize, const void* base, int64_t rows,
                      int64_t cols, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * esize) % 16) return cudaErrorMisalignedAddress;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Per device: SM count and whether each kernel's shared-memory limit was raised.
struct DevState {
  int sms = 0;
  bool attr[4] = {false, false, false, false};
};
DevState g_dev[64];
std::mutex g_dev_mu;

template <int NA, int NT, int GR, int EPI>
cudaError_t launch_tc(int slot, const __half* a_codes, int T, int K, const __half* w_codes, const float* ws,
                      int w_rows, const uint32_t* a_absmax, const int32_t* row_seq, float* c, uint32_t* out_absmax,
                      uint32_t* err, cudaStream_t stream) {
  using G = TileCfg<NA, NT, GR>;
  auto kern = gemm_q8_tc_kernel<NA, NT, GR, EPI>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int sms;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevState& ds = g_dev[dev];
    if (!ds.sms && (e = cudaDeviceGetAttribute(&ds.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    if (!ds.attr[slot]) {
      if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem)) != cudaSuccess)
        return e;
      ds.attr[slot] = true;
    }
    sms = ds.sms;
  }
  const int n_per_a = w_rows / NA;
  CUtensorMap tm_w, tm_a, tm_c;
  if ((e = encode_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w_codes, w_rows, K, kBKS, kBM,
                     CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
    return e;
  if ((e = encode_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_codes, T, K, kBKS, NT,
                     CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
    return e;
  if ((e = encode_2d(&tm_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, c, T, n_per_a, kBM, kSubTok,
                     CU_TENSOR_MAP_SWIZZLE_NONE)) != cudaSuccess)
    return e;
  const int total = (n_per_a / kBM) * ((T + NT - 1) / NT);
  const int grid = total < sms ? total : sms;
  kern<<<grid, G::kThreads, G::kSmem, stream>>>(tm_w, tm_a, tm_c, ws, w_rows, n_per_a, T, K, a_absmax, row_seq,
                                             out_absmax, err, c);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_q8(const __half* a_codes, const __half* w_codes, const float* w_scales, int M, int N, int K,
                           const uint32_t* a_absmax, const int32_t* row_seq, float* c, int epilogue,
                           uint32_t* out_absmax, uint32_t* err, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (M < 0 || K <= 0 || K % 128 != 0) return cudaErrorInvalidValue;  // four Q8_0 blocks per scale load
  if (epilogue == kEpiGeluUp) {
    if (N % (2 * kBM) != 0) return cudaErrorInvalidValue;
    return launch_tc<2, 96, 3, kEpiGeluUp>(0, a_codes, M, K, w_codes, w_scales, N, a_absmax, row_seq, c, out_absmax,
                                        err, stream);
  }
  if (N % kBM != 0) return cudaErrorInvalidValue;
  // small batches: narrower token tiles keep more SMs busy
  if ((N / kBM) * ((M + 191) / 192) < 148)
    return launch_tc<1, 96, 3, kEpiStore>(1, a_codes, M, K, w_codes, w_scales, N, a_absmax, row_seq, c, nullptr, err,
                                       stream);
  return launch_tc<1, 192, 3, kEpiStore>(2, a_codes, M, K, w_codes, w_scales, N, a_absmax, row_seq, c, nullptr, err,
                                      stream);
}

}  // namespace sem
