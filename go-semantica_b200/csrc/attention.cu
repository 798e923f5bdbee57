// Bidirectional GQA attention for EmbeddingGemma (runAttentionINT8 ->
// MultiHeadAttentionChunked, internal/runtime/model_int8.go:455-500,
// internal/kernels/attention.go:178-310, softmax activation.go:161-213) on the
// sm_100a tensor cores (tcgen05, accumulators in TMEM).
//
// The reference materialises the scores of every query row, takes the exact
// row max, applies its polynomial fastExp (which clamps arguments below -10 to
// zero) and multiplies by 1/sum. Because of that clamp an online-softmax
// rescale would change results, so the keys are visited twice:
//   pass 1: scores from the fp16 high halves only, to find each row's max;
//   pass 2: scores with three-term fp16 products (hi*hi + hi*lo + lo*hi, where
//           x = hi + lo to ~22 bits) for near-fp32 accuracy,
//           p = fastExp(score - max), row sums, and O += P V, again with
//           three-term products of split P and V.
// The max from pass 1 differs from the exact max by the fp16 error of one
// score; fastExp(x - d) = fastExp(x) * e^-d up to O(1e-3 d), and the common
// factor cancels in the normalisation.
//
// One CTA = 128 query rows of one (sequence, head), keys in tiles of 128.
// Q (hi and lo, 128 KB) stays in shared memory; K and V stream through a ring
// of three 32 KB slots, each filled by one 4-D TMA copy that lands both planes
// (hi, lo) of a piece: 128 keys x 64 dims of K, or 32 keys x 256 dims of V, so
// the MMAs consume one slot while the next two load.
// TMEM holds O (256 fp32 columns) and two 128-column score buffers, so the
// score MMAs are N = 128 (a kind::f16 MMA costs ~100 cycles whatever its N up
// to 128, so wider tiles do more work per instruction). The softmax writes P
// in place over the scores it has read (per 16 keys: 8 columns of p_hi then 8
// of p_lo, packed fp16 pairs); the P.V MMAs take A from TMEM and V MN-major
// with N = 256 (all dims at once), and a score buffer takes new scores once
// its P.V MMAs complete. Warps 0 and 2 issue TMA (alternate slots), warp 1 the
// MMAs, warps 4-11 (two per TMEM lane quarter, each half of a tile's keys) do
// the softmax with packed fp32 arithmetic and at the end scale O by 1/sum;
// full query tiles leave through swizzled shared-memory boxes (where Q was)
// and TMA stores. V is read MN-major straight from its row-major [token][dim]
// layout, so sequences may start at any token. All three query heads read the
// single KV head (GQA) through L2.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sem {

namespace {

constexpr int HD = 256;      // head_dim
constexpr int QT = 128;      // query rows per CTA (TMEM lanes)
constexpr int KT = 128;      // keys per tile (score MMAs of N = 128)
constexpr int NSLOT = 3;     // K/V ring slots
constexpr int SLOT = 32768;  // 32 KB slots (see the ring order below)
constexpr int PLANE = SLOT / 2;          // 16 KB: the hi or lo half of a pass-2 slot
constexpr int VKEYS = 32;                // keys per pass-2 V slot
constexpr int VDBLK = VKEYS * 128;       // 4 KB: one dim block of a V slot plane (32 keys x 128 B)
constexpr int DBLK1 = KT * 128;          // 16 KB: one dim block of a pass-1 K slot (128 keys x 128 B)
constexpr int OBOX = QT * 128;           // 16 KB: one 32-float x 128-row output box
constexpr int QBLK = QT * 128;           // 16 KB: 128 rows x 64 dims
constexpr int SMEM_Q = 2 * 4 * QBLK;     // hi, lo x 4 dim blocks: 128 KB
constexpr int SMEM_RING = NSLOT * SLOT;  // 96 KB
constexpr int NS1 = 2;  // score buffers of pass 1 (128 columns each, in the O columns, unused until pass 2)
// q, ring full/empty, S full, P full, S/P buffer free, O, drain, pass-1 S full/empty
constexpr int NBAR = 1 + 2 * NSLOT + 2 + 2 + 2 + 1 + 1 + 2 * NS1 + 1;
constexpr int BAR_BLOCK = 320;                     // barriers, TMEM address, abort flag
constexpr int SMEM_MISC = BAR_BLOCK + 2 * QT * 4;  // + [2][QT] reductions
constexpr int SMEM_BYTES = 1024 + SMEM_Q + SMEM_RING + SMEM_MISC;
constexpr int THREADS = 384;  // warpgroup 0: TMA (warps 0, 2), MMA (1), idle (3); warpgroups 1-2: softmax / epilogue
constexpr int SM_WARPS = 8;
// TMEM columns: O [0,256), score / P buffers [256,384) and [384,512)
constexpr uint32_t TM_O = 0, TM_S = 256;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(8 * OBOX <= SMEM_Q, "the output tile is staged where Q was");
static_assert(NBAR * 8 + 8 <= BAR_BLOCK, "barrier block");

__device__ uint32_t g_attn_error;

__device__ __forceinline__ void tmem_ld16_w(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }
__device__ __forceinline__ void tmem_wait_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] x B[smem]^T: A (M = 128 rows = TMEM lanes) packed two
// fp16 per 32-bit column along K.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same on an SM pair: M = 256 rows, A from both CTAs' TMEM at d/a, B
// halves in both CTAs' shared memory at the descriptor's offsets.
__device__ __forceinline__ void umma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand tile with 128-byte swizzle:
// rows of 128 bytes hold 64 consecutive MN elements, 8-row groups along K are
// 1024 bytes apart (SBO), and the next 64 MN elements sit `lbo` bytes further.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

}  // namespace

// WIN: sliding-window layers (model-faithful mode). The full-attention
// instances keep the window tests out of their score loops.
// PAIR: a cluster of two CTAs on an SM pair shares one 256-row query tile of
// a (sequence, head): CTA r owns rows [128 r, +128) (its Q, TMEM rows, softmax
// and output), and the leader's cta_group::2 MMAs (M = 256) read B halves from
// both CTAs: keys [64 r, +64) of each 128-key tile for the scores, dims
// [128 r, +128) of V for P.V. Each SM thus stages half the K/V bytes and reads
// 6 KB of shared memory per score MMA instead of 8 KB (shared-memory bandwidth
// bounds the single-SM kernel's N = 128 score MMAs). TMA copies of both CTAs
// complete on the leader's barriers; MMA commits reach both CTAs'.
template <bool WIN, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qh, const __grid_constant__ CUtensorMap tm_ql,
                        const __grid_constant__ CUtensorMap tm_k1, const __grid_constant__ CUtensorMap tm_k2,
                        const __grid_constant__ CUtensorMap tm_v2, const __grid_constant__ CUtensorMap tm_out, int nh,
                        float scale, int hw, SeqMeta meta, AttnTiles tiles, float* __restrict__ out,
                        uint32_t* __restrict__ absmax, uint32_t* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                      // [plane][dblock][128 rows x 128 B]
  uint8_t* sRing = sQ + SMEM_Q;            // [slot][2 boxes of 64 keys x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + SMEM_RING);
  uint64_t* qfull = bars;
  uint64_t* rfull = bars + 1;
  uint64_t* rempty = rfull + NSLOT;
  uint64_t* sfull = rempty + NSLOT;
  uint64_t* pfull = sfull + 2;
  uint64_t* pfree = pfull + 2;  // the P.V MMAs of a buffer completed: it may take new scores
  uint64_t* ofull = pfree + 2;
  uint64_t* drain = ofull + 1;
  uint64_t* s1full = drain + 1;
  uint64_t* s1empty = s1full + NS1;
  uint64_t* qlofull = s1empty + NS1;  // Q lo landed (pass 1 needs only Q hi, behind qfull)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_red = reinterpret_cast<float*>(sRing + SMEM_RING + BAR_BLOCK);  // [2 halves][QT]: maxima, later sums
  if (!err) err = &g_attn_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  // heads vary fastest, so the CTAs of one sequence (query tiles x heads) run
  // together and read its K and V from L2 rather than from DRAM
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile = unit / nh, head = unit % nh;
  const int seq = tiles.tile_seq[tile];
  const int row0 = tiles.tile_row0[tile] + (int)rank * QT;  // this CTA's query rows
  const int s_beg = meta.cu_seqlens[seq], s_end = meta.cu_seqlens[seq + 1];
  const int n_rows = min(QT, s_end - row0);
  const int n_keys = s_end - s_beg;
  // key tiles this query tile sees: all of them, or (a sliding-window layer,
  // query rows see keys within hw positions) the tiles its rows' windows
  // reach; every loop below walks nkt tiles from jlo
  const int q_pos0 = row0 - s_beg;
  const bool windowed = WIN && hw < n_keys;
  const int jlo = windowed ? max(0, q_pos0 - hw) / KT : 0;
  const int jhi = windowed ? min(n_keys - 1, q_pos0 + n_rows - 1 + hw) / KT : (n_keys - 1) / KT;
  const int nkt = n_keys > 0 ? jhi - jlo + 1 : 0;
  const int key0 = s_beg + jlo * KT;  // first key (token row) of tile 0 of the walk
  // pass 1 (row maxima) takes 256-key tiles on a pair (N = 256 MMAs into
  // O's columns and the two score buffers, all free until pass 2), 128-key
  // tiles on one CTA
  constexpr int KT1 = PAIR ? 2 * KT : KT;
  const int nkt1 = PAIR ? (n_keys + KT1 - 1) / KT1 : nkt;

  constexpr int NCTA = PAIR ? 2 : 1;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(&bars[i], 1);
    mbar_init(pfull, NCTA * SM_WARPS);  // (the leader's) both CTAs' softmax warps
    mbar_init(pfull + 1, NCTA * SM_WARPS);
    for (int k = 0; k < NS1; ++k) mbar_init(&s1empty[k], NCTA * SM_WARPS);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (PAIR)
      tmem_alloc_pair(s_tmem, 512);
    else
      tmem_alloc(s_tmem, 512);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // the leader's copy of one of this CTA's barriers (a shared::cluster address)
  const uint32_t lead_bars = PAIR ? mapa_shared(smem_u32(bars), 0) : smem_u32(bars);
  auto lbar = [&](const uint64_t* b) -> uint32_t {
    return lead_bars + (uint32_t)(reinterpret_cast<const uint8_t*>(b) - reinterpret_cast<const uint8_t*>(bars));
  };

  // Ring consumption order (128-key tiles): pass 1 = K hi of each tile, dims
  // 0-127 then 128-255 (two slots of [2 dim blocks][128 keys][128 B]); pass 2
  // = K(0), then for j = 1..: K(j), V(j-1); finally V(last). A K(j) item is
  // four slots, one per 64-dim block, each [hi, lo][128 keys][128 B]; a V(j)
  // item is four slots, one per 32 keys, each [hi, lo][4 dim blocks][32 keys]
  // [128 B]. Every pass-2 slot holds both planes its MMAs need, so the MMAs
  // work on one slot while the other two load.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;  // 128 x 88 + 256 x 192 <= 384 x 168");
    if ((warp == 0 || warp == 2) && lane == 0) {
      // ---------------- TMA producers ----------------
      // Two threads (warps 0 and 2) walk the same slot sequence and issue
      // alternate slots: one thread's loads complete at a limited rate (a few
      // copies in flight), so a second stream doubles the rate.
      const uint32_t me = warp >> 1;
      uint32_t it = 0;
      bool ok = true;
      // Q hi / Q lo of this CTA's rows (on a pair: completing on the leader's
      // barrier, which expects both CTAs' bytes)
      auto load_q = [&](const CUtensorMap* map, uint64_t* bar, uint8_t* dst) {
        if (PAIR) {
          if (rank == 0) mbar_arrive_expect_tx(bar, SMEM_Q);
#pragma unroll
          for (int b = 0; b < 4; ++b) tma_load_3d_pair(map, lbar(bar), dst + b * QBLK, b * 64, head, row0);
        } else {
          mbar_arrive_expect_tx(bar, SMEM_Q / 2);
#pragma unroll
          for (int b = 0; b < 4; ++b) tma_load_3d(map, bar, dst + b * QBLK, b * 64, head, row0);
        }
      };
      if (me == 0) load_q(&tm_qh, qfull, sQ);
      // one slot: a 3-D box (pass 1) or a 4-D box whose outermost dimension is
      // the plane (pass 2)
      auto load_slot = [&](const CUtensorMap* map, bool four, int row, int dblk0) -> bool {
        if ((it & 1) != me) {
          ++it;
          return true;
        }
        const uint32_t s = it % NSLOT, u = it / NSLOT;
        if (!mbar_wait(&rempty[s], (u & 1) ^ 1, abort_flag, err, 1u)) return false;
        if (PAIR) {
          if (rank == 0) mbar_arrive_expect_tx(&rfull[s], 2 * SLOT);
          if (four)
            tma_load_4d_pair(map, lbar(&rfull[s]), sRing + s * SLOT, 0, row, dblk0, 0);
          else
            tma_load_3d_pair(map, lbar(&rfull[s]), sRing + s * SLOT, 0, row, dblk0);
        } else {
          mbar_arrive_expect_tx(&rfull[s], SLOT);
          if (four)
            tma_load_4d(map, &rfull[s], sRing + s * SLOT, 0, row, dblk0, 0);  // 64 dims x rows x dim blocks x planes
          else
            tma_load_3d(map, &rfull[s], sRing + s * SLOT, 0, row, dblk0);  // 64 dims x rows x dim blocks
        }
        ++it;
        return true;
      };
      // On a pair every slot holds this CTA's half: keys [64 r, +64) of a
      // 128-key tile (K), or dims [128 r, +128) of 64 keys (V).
      const int khalf = PAIR ? 64 * (int)rank : 0;
      // pass 1: per key tile (KT1 keys; on a pair this CTA's half of 256)
      // two slots, [2 dim blocks][128 keys][128 B] each
      for (int j = 0; ok && j < nkt1; ++j) {
        for (int h = 0; ok && h < 2; ++h) ok = load_slot(&tm_k1, false, key0 + j * KT1 + 2 * khalf, 2 * h);
        if (j == 0 && me == 0) load_q(&tm_ql, qlofull, sQ + 4 * QBLK);  // Q lo behind the first K tile
      }
      if (nkt == 0 && me == 0) load_q(&tm_ql, qlofull, sQ + 4 * QBLK);  // keep the barrier's one phase complete
      for (int j = 0; ok && j <= nkt; ++j) {
        if (PAIR) {
          if (j < nkt)  // [hi, lo][2 dim blocks][64 keys][128 B], dim blocks 2h, 2h + 1
            for (int h = 0; ok && h < 2; ++h) ok = load_slot(&tm_k2, true, key0 + j * KT + khalf, 2 * h);
          if (j >= 1)  // [hi, lo][dim blocks 2r, 2r + 1][64 keys][128 B]
            for (int kq = 0; ok && kq < 2; ++kq)
              ok = load_slot(&tm_v2, true, key0 + (j - 1) * KT + 64 * kq, 2 * (int)rank);
        } else {
          if (j < nkt)
            for (int db = 0; ok && db < 4; ++db) ok = load_slot(&tm_k2, true, key0 + j * KT, db);
          if (j >= 1)
            for (int kq = 0; ok && kq < KT / VKEYS; ++kq)
              ok = load_slot(&tm_v2, true, key0 + (j - 1) * KT + kq * VKEYS, 0);
        }
      }
      // copies in flight land before shared memory is released (on a pair the
      // leader's barriers count both CTAs' bytes, and the final cluster
      // barrier keeps the peer alive until then)
      if (rank == 0) {
        for (uint32_t j = it > (uint32_t)NSLOT ? it - NSLOT : 0; j < it; ++j)
          if ((j & 1) == me) mbar_wait_drain(&rfull[j % NSLOT], (j / NSLOT) & 1);
        if (me == 0) {
          mbar_wait_drain(qfull, 0);
          mbar_wait_drain(qlofull, 0);
        }
      }
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ---------------- MMA issuer (on a pair: the leader's, for both SMs) ----------------
      constexpr uint32_t idesc_qk = umma_idesc_f16_f32(NCTA * QT, KT);  // N = 128 keys
      constexpr uint32_t idesc_pv = umma_idesc_f16_f32(NCTA * QT, HD) | (1u << 16);  // N = 256 dims, B (V) MN-major
      auto mma_ss = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
        if (PAIR)
          umma_f16_pair(d, a, b, idesc, acc);
        else
          umma_f16(d, a, b, idesc, acc);
      };
      auto mma_ts = [&](uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
        if (PAIR)
          umma_f16_ts_pair(d, a, b, idesc, acc);
        else
          umma_f16_ts(d, a, b, idesc, acc);
      };
      // completion of every MMA issued so far, signalled to both CTAs' (all)
      // or only this CTA's (lead) copy of a barrier
      auto commit_all = [&](uint64_t* bar) {
        if (PAIR)
          umma_commit_pair_mc(bar, 0x3);
        else
          umma_commit(bar);
      };
      auto commit_lead = [&](uint64_t* bar) {
        if (PAIR)
          umma_commit_pair_mc(bar, 0x1);
        else
          umma_commit(bar);
      };
      uint32_t it = 0, sfill = 0;
      bool ok = mbar_wait(qfull, 0, abort_flag, err, 2u);
      tc_fence_after();
      const uint32_t q_hi = smem_u32(sQ), q_lo = smem_u32(sQ + 4 * QBLK);
      auto take_slot = [&](uint32_t& addr) -> bool {
        const uint32_t s = it % NSLOT, u = it / NSLOT;
        if (!mbar_wait(&rfull[s], u & 1, abort_flag, err, 2u)) return false;
        tc_fence_after();
        addr = smem_u32(sRing + s * SLOT);
        return true;
      };
      auto free_slot = [&]() { commit_all(&rempty[it % NSLOT]); ++it; };
      // pass 1: S1[buf] = q_hi . k_hi of a tile; one CTA: NS1 128-column
      // buffers in the O columns; a pair: N = 256, buffer 0 in O's columns,
      // buffer 1 in the two score buffers' (pass 2 has not started)
      constexpr uint32_t idesc_qk1 = umma_idesc_f16_f32(NCTA * QT, KT1);
      uint32_t fill1 = 0;
      auto qk1 = [&]() -> bool {
        const uint32_t b = fill1 % NS1, ub = fill1 / NS1;
        if (!mbar_wait(&s1empty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) return false;
        const uint32_t d_s = PAIR ? tmem + (b ? TM_S : TM_O) : tmem + TM_O + b * KT;
        ++fill1;
        tc_fence_after();
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {  // dims 0-127, then 128-255: one slot each ([2 dim blocks][128 keys][128 B])
          uint32_t k_a;
          if (!take_slot(k_a)) return false;
#pragma unroll
          for (int k16 = 0; k16 < 8; ++k16) {
            const int db = 2 * h + k16 / 4;
            const uint32_t koff = (uint32_t)(k16 % 4) * 32;
            const uint32_t kb = (uint32_t)(k16 / 4) * DBLK1 + koff;
            mma_ss(d_s, umma_desc_k_sw128(q_hi + db * QBLK + koff), umma_desc_k_sw128(k_a + kb), idesc_qk1,
                   (h | k16) ? 1u : 0u);
          }
          free_slot();
        }
        commit_all(&s1full[b]);
        return true;
      };
      // pass 2: S[buf] (two buffers at TM_S) = three-term scores of a tile
      auto qk = [&]() -> bool {
        const uint32_t b = sfill & 1, ub = sfill >> 1;
        // the buffer's previous P.V MMAs have read its P (first use: no wait)
        if (!mbar_wait(&pfree[b], (ub & 1) ^ 1, abort_flag, err, 2u)) return false;
        const uint32_t d_s = tmem + TM_S + b * KT;
        ++sfill;
        tc_fence_after();
        if (PAIR) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {  // one slot per two 64-dim blocks: [hi, lo][2 dim blocks][64 keys][128 B]
            uint32_t k_a;
            if (!take_slot(k_a)) return false;
#pragma unroll
            for (int k16 = 0; k16 < 8; ++k16) {
              const int dbl = k16 / 4;
              const uint32_t koff = (uint32_t)(k16 % 4) * 32;
              const uint32_t qb = (uint32_t)(2 * h + dbl) * QBLK + koff;
              const uint32_t kb = (uint32_t)dbl * (64 * 128) + koff;
              mma_ss(d_s, umma_desc_k_sw128(q_hi + qb), umma_desc_k_sw128(k_a + kb), idesc_qk, (h | k16) ? 1u : 0u);
              mma_ss(d_s, umma_desc_k_sw128(q_hi + qb), umma_desc_k_sw128(k_a + SLOT / 2 + kb), idesc_qk, 1u);
              mma_ss(d_s, umma_desc_k_sw128(q_lo + qb), umma_desc_k_sw128(k_a + kb), idesc_qk, 1u);
            }
            free_slot();
          }
        } else {
#pragma unroll 1
          for (int db = 0; db < 4; ++db) {  // one slot per 64-dim block: [hi, lo][128 keys][128 B]
            uint32_t k_a;
            if (!take_slot(k_a)) return false;
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
              const uint32_t koff = (uint32_t)k16 * 32;  // K=16 slice within the 128-byte row
              const uint32_t qb = (uint32_t)db * QBLK + koff;
              mma_ss(d_s, umma_desc_k_sw128(q_hi + qb), umma_desc_k_sw128(k_a + koff), idesc_qk, (db | k16) ? 1u : 0u);
              mma_ss(d_s, umma_desc_k_sw128(q_hi + qb), umma_desc_k_sw128(k_a + PLANE + koff), idesc_qk, 1u);
              mma_ss(d_s, umma_desc_k_sw128(q_lo + qb), umma_desc_k_sw128(k_a + koff), idesc_qk, 1u);
            }
            free_slot();
          }
        }
        commit_all(&sfull[b]);
        return true;
      };
      // O += P(j) V(j), three terms
      auto pv = [&](int j) -> bool {
        const uint32_t pb = j & 1;
        if (!mbar_wait(&pfull[pb], (j >> 1) & 1, abort_flag, err, 2u)) return false;
        tc_fence_after();
        const uint32_t p_buf = tmem + TM_S + pb * KT;  // P written over the scores
        const uint32_t d_o = tmem + TM_O;
        // a slot holds `keys` keys: [hi, lo][dim blocks][keys][128 B]; per CTA
        // N = 256 dims (4 dim blocks VDBLK apart) or, on a pair, 128 (2 blocks)
        constexpr int keys = PAIR ? 64 : VKEYS;
        constexpr uint32_t lbo = PAIR ? 64 * 128 : VDBLK;
#pragma unroll 1
        for (int kq = 0; kq < KT / keys; ++kq) {
          uint32_t v_a;
          if (!take_slot(v_a)) return false;
#pragma unroll
          for (int k16 = 0; k16 < keys / 16; ++k16) {
            // keys (keys kq + 16 k16)..: p_hi in 8 packed fp16 columns, then p_lo in the next 8
            const uint32_t p_hi = p_buf + (uint32_t)(kq * (keys / 16) + k16) * 16, p_lo = p_hi + 8;
            const uint32_t voff = (uint32_t)k16 * 2048;  // two 8-key groups of V rows
            const uint32_t acc0 = (j > 0 || kq > 0 || k16 > 0) ? 1u : 0u;
            mma_ts(d_o, p_hi, umma_desc_mn_sw128(v_a + voff, lbo), idesc_pv, acc0);
            mma_ts(d_o, p_hi, umma_desc_mn_sw128(v_a + SLOT / 2 + voff, lbo), idesc_pv, 1u);
            mma_ts(d_o, p_lo, umma_desc_mn_sw128(v_a + voff, lbo), idesc_pv, 1u);
          }
          free_slot();
        }
        commit_lead(&pfree[pb]);
        return true;
      };
      for (int j = 0; ok && j < nkt1; ++j) ok = qk1();
      if (ok) ok = mbar_wait(qlofull, 0, abort_flag, err, 2u);
      // the softmax has read every pass-1 buffer before pass 2 writes the
      // score buffers (a pair) or P.V the O columns (one CTA)
      auto drained1 = [&]() -> bool {
        for (int k = 0; k < NS1 && k < nkt1; ++k) {
          const int last = k + NS1 * ((nkt1 - 1 - k) / NS1);
          if (!mbar_wait(&s1empty[k], (last / NS1) & 1, abort_flag, err, 2u)) return false;
        }
        return true;
      };
      if (PAIR && ok) ok = drained1();
      tc_fence_after();
      for (int j = 0; ok && j <= nkt; ++j) {
        if (j < nkt) ok = qk();
        if (!PAIR && ok && j == 1) ok = drained1();
        if (ok && j >= 1) ok = pv(j - 1);
      }
      commit_all(ofull);
      commit_lead(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;");
    // ---------------- softmax and epilogue ----------------
    // arrivals the MMA issuer waits for go to the leader's barrier on a pair
    // (the leader's own warps arrive locally: no cluster-scope release)
    auto arrive_lead = [&](uint64_t* b) {
      if (PAIR && rank != 0)
        mbar_arrive_cluster(lbar(b));
      else
        mbar_arrive(b);
    };
    const int w = warp - 4;
    const int q = warp & 3;       // TMEM lane quarter
    const int half = w >> 2;      // keys [64*half, 64*half + 64) of each tile; O columns [128*half, +128)
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    // key k (position within the sequence) counts for this row when it exists
    // and, in a sliding-window layer, lies within hw positions of the row
    const int qpos = q_pos0 + r;
    auto key_ok = [&](int k) { return k < n_keys && (!windowed || (k >= qpos - hw && k <= qpos + hw)); };
    uint32_t sfill = 0;
    bool ok = true;
    auto wait_s = [&](uint32_t& col) {
      const uint32_t b = sfill & 1, ub = sfill >> 1;
      if (ok) ok = mbar_wait(&sfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      col = TM_S + b * KT + half * 64;
    };
    // ---- pass 1: row max of the fp16 scores ----
    float m = -INFINITY;
    for (int j = 0; j < nkt1; ++j) {
      const uint32_t b = j % NS1;
      if (ok) ok = mbar_wait(&s1full[b], (j / NS1) & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      if (ok) {
        // this half's KT1 / 2 keys of the tile, 64 at a time
        const uint32_t col0 = PAIR ? (b ? TM_S : TM_O) + half * (KT1 / 2) : TM_O + b * KT + half * 64;
#pragma unroll 1
        for (int sub = 0; sub < KT1 / 128; ++sub) {
          uint32_t s[4][16];
          const uint32_t col = col0 + sub * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld16_w(t_lane + col + 16 * c, s[c]);
          tmem_wait_regs(s[0]);
          reg_barrier16(s[1]);
          reg_barrier16(s[2]);
          reg_barrier16(s[3]);
          if (sub + 1 == KT1 / 128) {  // every score of the buffer is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_lead(&s1empty[b]);
          }
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int key = (jlo * KT) + j * KT1 + half * (KT1 / 2) + sub * 64 + c;
            if (key_ok(key)) m = fmaxf(m, __fmul_rn(__uint_as_float(s[c >> 4][c & 15]), scale));
          }
        }
      } else {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_lead(&s1empty[b]);
      }
    }
    s_red[half * QT + r] = m;
    named_bar_sync(1, SM_WARPS * 32);
    m = fmaxf(s_red[r], s_red[QT + r]);
    // ---- pass 2: p = fastExp(s - max), row sums, P (split fp16) into TMEM ----
    uint64_t l2 = 0;  // two partial row sums (even and odd keys)
    const uint64_t scale2 = pack2(scale, scale), negm2 = pack2(-m, -m);
    for (int j = 0; j < nkt; ++j) {
      uint32_t col;
      wait_s(col);
      ++sfill;
      const uint32_t pb = j & 1;
#pragma unroll 1
      for (int sub = 0; ok && sub < 2; ++sub, col += 32) {  // this half's 64 keys, 32 at a time
        uint32_t s[2][16];
        tmem_ld16_w(t_lane + col, s[0]);
        tmem_ld16_w(t_lane + col + 16, s[1]);
        tmem_wait_regs(s[0]);
        reg_barrier16(s[1]);
        uint32_t ph[16], pl[16];  // 32 keys as packed fp16 pairs
        const int kbase = (jlo + j) * KT + half * 64 + sub * 32;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          // score *= scale (attention.go:300), then fastExp(score - max)
          const uint64_t sc = mul2(pack2u(s[c >> 4][c & 15], s[c >> 4][(c & 15) + 1]), scale2);
          uint64_t p2 = fast_exp_ref2(add2(sc, negm2));
          if (windowed || kbase + c + 1 >= n_keys) {  // keys past the sequence end or the window weigh nothing
            float a, b;
            unpack2(p2, a, b);
            p2 = pack2(key_ok(kbase + c) ? a : 0.0f, key_ok(kbase + c + 1) ? b : 0.0f);
          }
          l2 = add2(l2, p2);
          float a, b;
          unpack2(p2, a, b);
          const __half2 hi = __floats2half2_rn(a, b);
          const float2 back = __half22float2(hi);
          const __half2 lo = __floats2half2_rn(__fsub_rn(a, back.x), __fsub_rn(b, back.y));
          ph[c >> 1] = *reinterpret_cast<const uint32_t*>(&hi);
          pl[c >> 1] = *reinterpret_cast<const uint32_t*>(&lo);
        }
        // P over the scores just read: per 16 keys, 8 columns of p_hi then 8 of p_lo
        uint32_t w0[16], w1[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          w0[i] = ph[i];
          w0[8 + i] = pl[i];
          w1[i] = ph[8 + i];
          w1[8 + i] = pl[8 + i];
        }
        tmem_st16(t_lane + col, w0);
        tmem_st16(t_lane + col + 16, w1);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_lead(&pfull[pb]);
    }
    float l0, l1;
    unpack2(l2, l0, l1);
    const float l = __fadd_rn(l0, l1);
    // ---- epilogue: O / sum, store, absmax ----
    named_bar_sync(1, SM_WARPS * 32);  // every thread has read its row max from s_red
    s_red[half * QT + r] = l;
    if (ok) ok = mbar_wait(ofull, 0, abort_flag, err, 8u);
    ok = __all_sync(0xffffffffu, ok);
    named_bar_sync(1, SM_WARPS * 32);
    tc_fence_after();
    const float lt = __fadd_rn(s_red[r], s_red[QT + r]);
    const float inv = lt > 0.0f ? __fdiv_rn(1.0f, lt) : 0.0f;
    const bool valid = r < n_rows;
    float amax = 0.0f;
    if (ok && n_rows == QT) {
      // A full tile leaves through shared memory (where Q was) and TMA
      // stores of 32-float x 128-row boxes in the 128-byte swizzled layout, so
      // the writes reach memory coalesced. Box (half * 4 + seg) holds dims
      // [32 (half * 4 + seg), +32); row r's 16-byte chunk k sits at chunk
      // k ^ (r & 7) of its 128-byte row.
#pragma unroll 1
      for (int seg = 0; seg < 4; ++seg) {
        uint32_t o[2][16];
        tmem_ld16_w(t_lane + TM_O + half * 128 + seg * 32, o[0]);
        tmem_ld16_w(t_lane + TM_O + half * 128 + seg * 32 + 16, o[1]);
        tmem_wait_regs(o[0]);
        reg_barrier16(o[1]);
        uint8_t* box = sQ + (half * 4 + seg) * OBOX + r * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[i] = __fmul_rn(__uint_as_float(o[k >> 2][(k & 3) * 4 + i]), inv);
            amax = fmaxf(amax, fabsf(v[i]));
          }
          *reinterpret_cast<float4*>(box + ((k ^ (r & 7)) << 4)) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, SM_WARPS * 32);
      if (warp == 4 && lane == 0) {
        for (int bx = 0; bx < 8; ++bx) tma_store_2d(&tm_out, sQ + bx * OBOX, head * HD + bx * 32, row0);
        bulk_commit();
        bulk_wait_all();  // the stores have read shared memory before the CTA exits
      }
      amax = warp_max(amax);
      if (lane == 0 && absmax) atomicMax(&absmax[seq], __float_as_uint(amax));
    } else {
    float* dst = out + (int64_t)(row0 + (valid ? r : 0)) * (nh * HD) + head * HD + half * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t o[16];
      if (ok) {
        tmem_ld16_w(t_lane + TM_O + half * 128 + c * 16, o);
        tmem_wait_regs(o);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0u;
      }
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = __fmul_rn(__uint_as_float(o[i]), inv);
        amax = fmaxf(amax, fabsf(v[i]));
      }
      if (valid) {
        float4* d4 = reinterpret_cast<float4*>(dst + c * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
    amax = warp_max(valid ? amax : 0.0f);
    if (lane == 0 && absmax) atomicMax(&absmax[seq], __float_as_uint(amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  // on a pair: the leader's MMAs have drained and no copy or arrival is still
  // aimed at either CTA
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, 512);
    else
      tmem_dealloc(tmem, 512);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 attn_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// fp16 row-major [rows][256] with a box of 64 x box_rows, 128-byte swizzle.
// k / v planes [rows][256] as a 3-D map (64 dims, row, dim block of 64) with
// a box of 64 x box_rows x box_dblks: one copy lands box_dblks 128-byte-wide
// dim blocks of box_rows rows one after another, each in the 128-byte
// swizzled K-major layout.
cudaError_t map_rows(CUtensorMap* m, const __half* base, int64_t rows, int box_rows, int box_dblks) {
  auto enc = attn_encoder();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15) return cudaErrorMisalignedAddress;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(HD / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)HD * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_dblks};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

// k or v hi and lo planes [2][rows][256] (lo right after hi) as a 4-D map
// (64 dims, row, dim block, plane) with a box of 64 x box_rows x box_dblks x 2:
// one copy lands [plane][dim block][row][128 B], each dim block in the
// 128-byte swizzled layout.
cudaError_t map_rows_pair(CUtensorMap* m, const __half* base, int64_t rows, int box_rows, int box_dblks) {
  auto enc = attn_encoder();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15) return cudaErrorMisalignedAddress;
  cuuint64_t dims[4] = {64, (cuuint64_t)rows, (cuuint64_t)(HD / 64), 2};
  cuuint64_t strides[3] = {(cuuint64_t)HD * 2, 128, (cuuint64_t)rows * HD * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_dblks, 2};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

// q planes [T][nh][256]: 3-D map (dim, head, token) with a box of 64 x 1 x 128.
cudaError_t map_q(CUtensorMap* m, const __half* base, int64_t T, int nh) {
  auto enc = attn_encoder();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15) return cudaErrorMisalignedAddress;
  cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)nh, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)nh * HD * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)QT};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

bool g_attn_attr[64];
std::mutex g_attn_mu;

}  // namespace

cudaError_t launch_attention(const __half* qh, const __half* ql, const __half* kh, const __half* kl, const __half* vh,
                             const __half* vl, int num_heads, float scale, int half_window, SeqMeta meta,
                             AttnTiles tiles, AttnTiles pair_tiles, float* out, uint32_t* absmax, uint32_t* err,
                             cudaStream_t stream) {
  const bool windowed = half_window > 0 && half_window < (1 << 24);
  const bool pair = !windowed && pair_tiles.n_tiles > 0;
  if ((pair ? pair_tiles.n_tiles : tiles.n_tiles) == 0) return cudaSuccess;
  const int64_t T = meta.T;
  CUtensorMap m_qh, m_ql, m_k1, m_k2, m_v2, m_out;
  cudaError_t e;
  // the lo plane of K and of V directly follows its hi plane (one 4-D map covers both)
  if (kl != kh + T * HD || vl != vh + T * HD) return cudaErrorInvalidValue;
  if ((e = map_q(&m_qh, qh, T, num_heads)) != cudaSuccess) return e;
  if ((e = map_q(&m_ql, ql, T, num_heads)) != cudaSuccess) return e;
  // One CTA: pass 1 K hi, 128 keys x 2 dim blocks; pass 2 K hi+lo, 128 keys x
  // 1 dim block; V hi+lo, 32 keys x 4 dim blocks. A pair's CTA: pass 1 K hi,
  // 128 keys (its half of 256) x 2 dim blocks; pass 2 K hi+lo, 64 keys x 2
  // dim blocks; V hi+lo, 64 keys x 2 dim blocks. 32 KB per copy in every case.
  if ((e = map_rows(&m_k1, kh, T, KT, 2)) != cudaSuccess) return e;
  if ((e = map_rows_pair(&m_k2, kh, T, pair ? 64 : KT, pair ? 2 : 1)) != cudaSuccess) return e;
  if ((e = map_rows_pair(&m_v2, vh, T, pair ? 64 : VKEYS, pair ? 2 : 4)) != cudaSuccess) return e;
  {  // out [T][nh * 256] fp32: boxes of 32 floats x 128 rows, 128-byte swizzle
    auto enc = attn_encoder();
    if (!enc) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(out) & 15) return cudaErrorMisalignedAddress;
    cuuint64_t dims[2] = {(cuuint64_t)num_heads * HD, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)num_heads * HD * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)QT};
    cuuint32_t es[2] = {1, 1};
    if (enc(&m_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(g_attn_mu);
    if (dev >= 0 && dev < 64 && !g_attn_attr[dev]) {
      if ((e = cudaFuncSetAttribute(attention_tc_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES)) != cudaSuccess ||
          (e = cudaFuncSetAttribute(attention_tc_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES)) != cudaSuccess ||
          (e = cudaFuncSetAttribute(attention_tc_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES)) != cudaSuccess)
        return e;
      g_attn_attr[dev] = true;
    }
  }
  if (pair) {  // clusters of two CTAs: 256-row query tiles
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pair_tiles.n_tiles * num_heads);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attention_tc_kernel<false, true>, m_qh, m_ql, m_k1, m_k2, m_v2, m_out, num_heads,
                              scale, 1 << 24, meta, pair_tiles, out, absmax, err);
  }
  dim3 grid(tiles.n_tiles * num_heads);
  if (windowed)
    attention_tc_kernel<true, false><<<grid, THREADS, SMEM_BYTES, stream>>>(
        m_qh, m_ql, m_k1, m_k2, m_v2, m_out, num_heads, scale, half_window, meta, tiles, out, absmax, err);
  else
    attention_tc_kernel<false, false><<<grid, THREADS, SMEM_BYTES, stream>>>(
        m_qh, m_ql, m_k1, m_k2, m_v2, m_out, num_heads, scale, 1 << 24, meta, tiles, out, absmax, err);
  return cudaGetLastError();
}

}  // namespace sem
