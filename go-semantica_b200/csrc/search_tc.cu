// search/brute exact scan on the sm_100a tensor cores (Index.searchNormalized,
// search/brute/index.go:55-154, under the integer contract: the query is
// quantised like the stored rows, quant.go:17-41, and scores are exact int32
// dot products).
//
// int8 rows x int8 queries on tcgen05.mma.kind::i8 with int32 accumulators in
// TMEM: the scores are exact, as in the CUDA-core scan. One CTA = 128 queries
// (TMEM lanes, the query codes resident in shared memory) x one contiguous part
// of the corpus, streamed as 256-row tiles through a TMA ring of 128-byte K
// slices; TMEM holds two score tiles so the MMAs of tile t+1 overlap the
// top-k filter of tile t. Warps 0 and 2 issue TMA (alternate stages), warp 1
// the MMAs, warps 4-11 (two per TMEM lane quarter, each half of a tile's rows)
// keep a per-query top-16 in registers: rows arrive in ascending order, so a candidate only enters
// when its score is strictly above the k-th best (a tie never beats a lower
// row). The k-th best score of each stream is also published, to the other
// half through shared memory and to the CTAs of later corpus parts through a
// per-query word in global memory; a row scoring below any published bound
// cannot reach the final top-k (k real rows beat it), so each 16-score chunk
// is usually rejected by one max-and-compare. The two halves merge in shared
// memory and emit one list of k keys per (query, part), padded with empty (0)
// keys; topk_merge_kernel merges the parts. CTAs are numbered part-major, so
// the query tiles that read one corpus part run together and share it
// through L2.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sem {

namespace {

constexpr int SQ = 128;                 // queries per CTA
constexpr int SN = 256;                 // corpus rows per tile
constexpr int SKB = 128;                // K bytes per stage / query box
constexpr int S_TILE = SN * SKB;        // 32 KB
constexpr int S_QBOX = SQ * SKB;        // 16 KB
constexpr int S_THREADS = 384;
constexpr int S_EPI_WARPS = 8;
constexpr int S_KMAX = 16;
constexpr int S_MAX_QBOX = 8;           // D <= 1024
constexpr int S_BAR_BYTES = 256;
constexpr int S_THR_BYTES = SQ * 4;     // per-query shared score bound

__device__ uint32_t g_search_error;

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::i8: signed A and B, s32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// kind::i8 with the signedness of each operand chosen: s8 (true) or u8 (false).
__host__ __device__ constexpr uint32_t idesc_i8s(int M, int N, bool a_signed, bool b_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// (bit b of x) ? hi : lo, opaque to the optimiser so that the select tree
// below is not turned back into an indexed (local-memory) array access.
__device__ __forceinline__ uint32_t sel_bit(uint32_t x, uint32_t b, uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "selp.b32 %0, %2, %3, p;\n\t}\n"
      : "=r"(r)
      : "r"(x & b), "r"(hi), "r"(lo));
  return r;
}

// sc[x] for a lane-varying x without local memory: a 4-level select tree.
__device__ __forceinline__ uint32_t pick16(const uint32_t (&sc)[16], uint32_t x) {
  uint32_t a[8], c[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = sel_bit(x, 1, sc[2 * i], sc[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = sel_bit(x, 2, a[2 * i], a[2 * i + 1]);
  return sel_bit(x, 8, sel_bit(x, 4, c[0], c[1]), sel_bit(x, 4, c[2], c[3]));
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Top16 {
  uint64_t v[S_KMAX];  // best first; 0 = empty
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < S_KMAX; ++i) v[i] = 0;
  }
  // The k-th best key (1 <= k <= 16), 0 while fewer than k are held.
  __device__ __forceinline__ uint64_t kth(int k) const {
    uint64_t r = v[0];
#pragma unroll
    for (int i = 1; i < S_KMAX; ++i) {  // opaque selects: no indexed (local-memory) access of v
      asm("{\n\t.reg .pred p;\n\t"
          "setp.eq.s32 p, %2, %3;\n\t"
          "selp.b64 %0, %1, %0, p;\n\t}\n"
          : "+l"(r)
          : "l"(v[i]), "r"(k - 1), "r"(i));
    }
    return r;
  }
  __device__ __forceinline__ void insert(uint64_t key) {
    v[S_KMAX - 1] = key;
#pragma unroll
    for (int i = S_KMAX - 1; i > 0; --i)
      if (v[i] > v[i - 1]) {
        const uint64_t t = v[i];
        v[i] = v[i - 1];
        v[i - 1] = t;
      }
  }
};

// One chunk of 16 scores of rows [row0, row0 + 16): the lane maximum rejects
// the chunk in the common case; otherwise the rows above thr enter one by one.
__device__ __forceinline__ void filter_chunk(const uint32_t (&sc)[16], int64_t row0, int64_t r1, int64_t row_base,
                                             bool live, int k, uint32_t ext, uint32_t& thr, uint32_t& own,
                                             Top16& top) {
  const int m = max(max(__vimax3_s32((int)sc[0], (int)sc[1], (int)sc[2]),
                        __vimax3_s32((int)sc[3], (int)sc[4], (int)sc[5])),
                    max(__vimax3_s32((int)sc[6], (int)sc[7], (int)sc[8]),
                        max(__vimax3_s32((int)sc[9], (int)sc[10], (int)sc[11]),
                            __vimax3_s32((int)sc[12], (int)sc[13], max((int)sc[14], (int)sc[15])))));
  if (!live || ((uint32_t)m ^ 0x80000000u) <= thr) return;
  uint32_t mask = 0;
#pragma unroll
  for (int x = 0; x < 16; ++x) mask |= (uint32_t)((sc[x] ^ 0x80000000u) > thr) << x;
  while (mask) {
    const uint32_t x = __ffs(mask) - 1;
    mask &= mask - 1;
    const uint32_t biased = pick16(sc, x) ^ 0x80000000u;
    const int64_t row = row0 + x;
    if (biased > thr && row < r1) {
      top.insert(((uint64_t)biased << 32) | (uint64_t)(0xffffffffu - (uint32_t)(row_base + row)));
      own = (uint32_t)(top.kth(k) >> 32);
      thr = max(own, ext ? ext - 1u : 0u);
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(S_THREADS, 1)
    search_tc_kernel(const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_q,
                     int64_t count, int nqb, int nst, int nq, int k, int64_t rows_per_part, int n_qtiles,
                     int n_parts, int64_t row_base, uint64_t* __restrict__ cand, uint32_t* __restrict__ qthr,
                     uint32_t* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                    // nqb boxes of 128 queries x 128 bytes
  uint8_t* sRing = sQ + nqb * S_QBOX;    // nst tiles of 256 rows x 128 bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + nst * S_TILE);
  uint64_t* qfull = bars;
  uint64_t* rfull = bars + 1;
  uint64_t* rempty = rfull + 4;
  uint64_t* tfull = rempty + 4;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile uint32_t* s_thr = reinterpret_cast<volatile uint32_t*>(reinterpret_cast<uint8_t*>(bars) + S_BAR_BYTES);
  if (!err) err = &g_search_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = blockIdx.x / n_qtiles, qt = blockIdx.x % n_qtiles;
  const int64_t r0 = (int64_t)part * rows_per_part;
  const int64_t r1 = min(count, r0 + rows_per_part);
  const int ntiles = r0 < r1 ? (int)((r1 - r0 + SN - 1) / SN) : 0;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], S_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < SQ) s_thr[threadIdx.x] = 0;
  if (warp == 1) tmem_alloc(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    if ((warp == 0 || warp == 2) && lane == 0) {
      // ---------------- TMA producers ----------------
      // Two threads (warps 0 and 2) issue alternate ring iterations: one
      // thread's stream of tile loads completes at about one stage per
      // microsecond, so two streams double the L2 -> SM rate of the SM.
      const uint32_t me = warp >> 1;
      if (me == 0) {
        mbar_arrive_expect_tx(qfull, nqb * S_QBOX);
        for (int b = 0; b < nqb; ++b) tma_load_2d(&tm_q, qfull, sQ + b * S_QBOX, b * SKB, qt * SQ);
      }
      uint32_t it = 0;
      bool ok = true;
      for (int t = 0; ok && t < ntiles; ++t)
        for (int b = 0; b < nqb; ++b, ++it) {
          if ((it & 1) != me) continue;
          const uint32_t s = it % nst, u = it / nst;
          if (!mbar_wait(&rempty[s], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&rfull[s], S_TILE);
          tma_load_2d(&tm_c, &rfull[s], sRing + s * S_TILE, b * SKB, (int)(r0 + (int64_t)t * SN));
        }
      // `it` is one past the last iteration this thread issued or skipped
      for (uint32_t j = it > (uint32_t)nst ? it - nst : 0; j < it; ++j)
        if ((j & 1) == me) mbar_wait_drain(&rfull[j % nst], (j / nst) & 1);
      if (me == 0) mbar_wait_drain(qfull, 0);
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_i8(SQ, SN);
      bool ok = mbar_wait(qfull, 0, abort_flag, err, 2u);
      tc_fence_after();
      const uint32_t q0 = smem_u32(sQ);
      uint32_t it = 0;
      for (int t = 0; ok && t < ntiles; ++t) {
        const uint32_t b = t & 1, ub = t >> 1;
        if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nqb; ++kb, ++it) {
          const uint32_t s = it % nst, u = it / nst;
          if (!mbar_wait(&rfull[s], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ca = smem_u32(sRing + s * S_TILE);
#pragma unroll
          for (int k32 = 0; k32 < SKB / 32; ++k32)
            umma_i8(tmem + b * SN, umma_desc_k_sw128(q0 + kb * S_QBOX + k32 * 32),
                    umma_desc_k_sw128(ca + k32 * 32), idesc, (kb | k32) ? 1u : 0u);
          umma_commit(&rempty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      umma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 152;");
    // ---------------- top-k filter ----------------
    const int w = warp - 4;
    const int q = warp & 3;     // TMEM lane quarter
    const int half = w >> 2;    // rows [128 * half, +128) of each tile
    const int lq = q * 32 + lane;  // query within the tile
    const int64_t qg = (int64_t)qt * SQ + lq;
    const bool live = qg < nq;
    const bool warp_live = __any_sync(0xffffffffu, live);
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t* gthr = (qthr && live) ? qthr + qg : nullptr;
    Top16 top;
    top.init();
    // Score bounds, as order-preserving (biased) score bits. own: the k-th
    // best score of this stream (0 while it holds fewer than k). ext: the
    // best k-th score published for this query by the other half of the
    // tile (shared memory) or by other corpus parts (global memory). Each is
    // the k-th best of k real rows, so a row whose score is below it cannot
    // reach the final top-k; a row tying it can (lower row wins), so ties
    // with ext are kept, and ties with own lose (rows arrive ascending).
    uint32_t own = 0, ext = gthr ? ld_relaxed_u32(gthr) : 0u, pub = 0;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t b = t & 1, ub = t >> 1;
      if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      if (!warp_live) {  // no real query in this lane quarter: nothing to read
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        continue;
      }
      ext = max(ext, s_thr[lq]);
      if (gthr && (t & 7) == 0) ext = max(ext, ld_relaxed_u32(gthr));
      uint32_t thr = max(own, ext ? ext - 1u : 0u);  // a row enters when its biased score > thr
      const int64_t rbase = r0 + (int64_t)t * SN + half * 128;
      // scores of 128 rows: 4 steps of two 16-column loads in flight
#pragma unroll 1
      for (int cp = 0; cp < 4; ++cp) {
        uint32_t sc[2][16];
        tmem_ld16(t_lane + b * SN + half * 128 + cp * 32, sc[0]);
        tmem_ld16(t_lane + b * SN + half * 128 + cp * 32 + 16, sc[1]);
        wait_ld16(sc[0]);
        reg_barrier16(sc[1]);
        if (cp == 3) {  // every score of this buffer is in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
        const uint32_t own0 = own;
        filter_chunk(sc[0], rbase + cp * 32, r1, row_base, live, k, ext, thr, own, top);
        filter_chunk(sc[1], rbase + cp * 32 + 16, r1, row_base, live, k, ext, thr, own, top);
        if (own != own0) atomicMax(const_cast<uint32_t*>(&s_thr[lq]), own);
      }
      if (gthr && own > pub && ((t & 7) == 7 || t == ntiles - 1)) {
        atomicMax(gthr, own);
        pub = own;
      }
    }
    // both halves of each query -> one list of k keys per (query, part)
    named_bar_sync(1, S_EPI_WARPS * 32);  // every tile consumed: the ring is free for the merge
    uint64_t* sk = reinterpret_cast<uint64_t*>(sRing);  // [SQ][S_KMAX], half 1's lists
    if (half == 1) {
#pragma unroll
      for (int i = 0; i < S_KMAX; ++i) sk[lq * S_KMAX + i] = top.v[i];
    }
    named_bar_sync(1, S_EPI_WARPS * 32);
    if (half == 0 && live) {
      uint64_t* dst = cand + ((int64_t)qg * n_parts + part) * k;
      const uint64_t* other = sk + lq * S_KMAX;
      int ib = 0;
      for (int i = 0; i < k; ++i) {
        const uint64_t bk = ib < S_KMAX ? other[ib] : 0;
        if (top.v[0] >= bk) {  // keys are unique except empty (0) entries
          dst[i] = top.v[0];
#pragma unroll
          for (int j = 0; j < S_KMAX - 1; ++j) top.v[j] = top.v[j + 1];
          top.v[S_KMAX - 1] = 0;
        } else {
          dst[i] = bk;
          ++ib;
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

// ---------------------------------------------------------------------------
// int16 rows x int16 queries (quant.go:110-135 under the integer contract):
// each code splits exactly into a signed high byte and an unsigned low byte,
// c = 256 * (c >> 8) + (c & 255), so
//   q . v = 65536 * (qh . vh) + 256 * (qh . vl + ql . vh) + (ql . vl),
// four kind::i8 products (per-operand signedness in the instruction
// descriptor) into three int32 TMEM accumulators. Each accumulator is exact
// (|qh . vh| <= 128^2 D, |ql . vl| <= 255^2 D), and the recombination in
// 32-bit two's complement arithmetic is exact because the true score fits in
// int32 (|q . v| <= |q| |v| < 2^31 for rows and queries of norm 1 scaled by
// 32767). The corpus and the queries are stored as byte planes (hi, lo) of
// D-byte rows. A tile is 64 rows, so two tiles' three accumulators (2 x 3 x 64
// columns) fit in TMEM; both query planes stay in shared memory (D <= 768),
// and the ring carries the two corpus planes' 128-byte K slices. The filter
// and the bounds are the int8 kernel's.
// ---------------------------------------------------------------------------
constexpr int SN16 = 64;                  // corpus rows per tile
constexpr int S16_SLICE = SN16 * SKB;     // 8 KB: one plane's K slice of a tile
constexpr int S16_STAGE = 2 * S16_SLICE;  // hi and lo planes
constexpr int S16_MAX_QBOX = 6;           // D <= 768
constexpr int S16_COLS = 3 * SN16;        // accumulators hh, cross, ll of one tile

__global__ void __launch_bounds__(S_THREADS, 1)
    search_tc16_kernel(const __grid_constant__ CUtensorMap tm_ch, const __grid_constant__ CUtensorMap tm_cl,
                       const __grid_constant__ CUtensorMap tm_qh, const __grid_constant__ CUtensorMap tm_ql,
                       int64_t count, int nqb, int nst, int nq, int k, int64_t rows_per_part, int n_qtiles,
                       int n_parts, int64_t row_base, uint64_t* __restrict__ cand, uint32_t* __restrict__ qthr,
                       uint32_t* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQh = smem;                    // nqb boxes of 128 queries x 128 bytes (high bytes)
  uint8_t* sQl = sQh + nqb * S_QBOX;      // the low bytes
  uint8_t* sRing = sQl + nqb * S_QBOX;    // nst stages of {hi slice, lo slice} of 64 rows x 128 bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + nst * S16_STAGE);
  uint64_t* qfull = bars;
  uint64_t* rfull = bars + 1;
  uint64_t* rempty = rfull + 4;
  uint64_t* tfull = rempty + 4;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile uint32_t* s_thr = reinterpret_cast<volatile uint32_t*>(reinterpret_cast<uint8_t*>(bars) + S_BAR_BYTES);
  if (!err) err = &g_search_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = blockIdx.x / n_qtiles, qt = blockIdx.x % n_qtiles;
  const int64_t r0 = (int64_t)part * rows_per_part;
  const int64_t r1 = min(count, r0 + rows_per_part);
  const int ntiles = r0 < r1 ? (int)((r1 - r0 + SN16 - 1) / SN16) : 0;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], S_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < SQ) s_thr[threadIdx.x] = 0;
  if (warp == 1) tmem_alloc(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    if ((warp == 0 || warp == 2) && lane == 0) {
      // ---------------- TMA producers (alternate ring iterations) ----------------
      const uint32_t me = warp >> 1;
      if (me == 0) {
        mbar_arrive_expect_tx(qfull, 2 * nqb * S_QBOX);
        for (int b = 0; b < nqb; ++b) {
          tma_load_2d(&tm_qh, qfull, sQh + b * S_QBOX, b * SKB, qt * SQ);
          tma_load_2d(&tm_ql, qfull, sQl + b * S_QBOX, b * SKB, qt * SQ);
        }
      }
      uint32_t it = 0;
      bool ok = true;
      for (int t = 0; ok && t < ntiles; ++t)
        for (int b = 0; b < nqb; ++b, ++it) {
          if ((it & 1) != me) continue;
          const uint32_t s = it % nst, u = it / nst;
          if (!mbar_wait(&rempty[s], (u & 1) ^ 1, abort_flag, err, 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&rfull[s], S16_STAGE);
          const int row = (int)(r0 + (int64_t)t * SN16);
          tma_load_2d(&tm_ch, &rfull[s], sRing + s * S16_STAGE, b * SKB, row);
          tma_load_2d(&tm_cl, &rfull[s], sRing + s * S16_STAGE + S16_SLICE, b * SKB, row);
        }
      for (uint32_t j = it > (uint32_t)nst ? it - nst : 0; j < it; ++j)
        if ((j & 1) == me) mbar_wait_drain(&rfull[j % nst], (j / nst) & 1);
      if (me == 0) mbar_wait_drain(qfull, 0);
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t id_hh = idesc_i8s(SQ, SN16, true, true);
      constexpr uint32_t id_hl = idesc_i8s(SQ, SN16, true, false);
      constexpr uint32_t id_lh = idesc_i8s(SQ, SN16, false, true);
      constexpr uint32_t id_ll = idesc_i8s(SQ, SN16, false, false);
      bool ok = mbar_wait(qfull, 0, abort_flag, err, 2u);
      tc_fence_after();
      const uint32_t qh0 = smem_u32(sQh), ql0 = smem_u32(sQl);
      uint32_t it = 0;
      for (int t = 0; ok && t < ntiles; ++t) {
        const uint32_t b = t & 1, ub = t >> 1;
        if (!mbar_wait(&tempty[b], (ub & 1) ^ 1, abort_flag, err, 2u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_hh = tmem + b * S16_COLS, d_x = d_hh + SN16, d_ll = d_hh + 2 * SN16;
        for (int kb = 0; kb < nqb; ++kb, ++it) {
          const uint32_t s = it % nst, u = it / nst;
          if (!mbar_wait(&rfull[s], u & 1, abort_flag, err, 2u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ch = smem_u32(sRing + s * S16_STAGE), cl = ch + S16_SLICE;
#pragma unroll
          for (int k32 = 0; k32 < SKB / 32; ++k32) {
            const uint32_t first = (kb | k32) ? 1u : 0u;
            const uint64_t aqh = umma_desc_k_sw128(qh0 + kb * S_QBOX + k32 * 32);
            const uint64_t aql = umma_desc_k_sw128(ql0 + kb * S_QBOX + k32 * 32);
            const uint64_t bvh = umma_desc_k_sw128(ch + k32 * 32), bvl = umma_desc_k_sw128(cl + k32 * 32);
            umma_i8(d_hh, aqh, bvh, id_hh, first);
            umma_i8(d_x, aqh, bvl, id_hl, first);
            umma_i8(d_x, aql, bvh, id_lh, 1u);
            umma_i8(d_ll, aql, bvl, id_ll, first);
          }
          umma_commit(&rempty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      umma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 152;");
    // ---------------- top-k filter ----------------
    const int w = warp - 4;
    const int q = warp & 3;        // TMEM lane quarter
    const int half = w >> 2;       // rows [32 * half, +32) of each tile
    const int lq = q * 32 + lane;  // query within the tile
    const int64_t qg = (int64_t)qt * SQ + lq;
    const bool live = qg < nq;
    const bool warp_live = __any_sync(0xffffffffu, live);
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t* gthr = (qthr && live) ? qthr + qg : nullptr;
    Top16 top;
    top.init();
    uint32_t own = 0, ext = gthr ? ld_relaxed_u32(gthr) : 0u, pub = 0;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t b = t & 1, ub = t >> 1;
      if (ok) ok = mbar_wait(&tfull[b], ub & 1, abort_flag, err, 4u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      if (!warp_live) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        continue;
      }
      ext = max(ext, s_thr[lq]);
      if (gthr && (t & 31) == 0) ext = max(ext, ld_relaxed_u32(gthr));
      uint32_t thr = max(own, ext ? ext - 1u : 0u);
      const int64_t rbase = r0 + (int64_t)t * SN16 + half * 32;
      const uint32_t col = t_lane + b * S16_COLS + half * 32;
      uint32_t hh[2][16], xx[2][16], ll[2][16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld16(col + c * 16, hh[c]);
        tmem_ld16(col + SN16 + c * 16, xx[c]);
        tmem_ld16(col + 2 * SN16 + c * 16, ll[c]);
      }
      wait_ld16(hh[0]);
      reg_barrier16(hh[1]);
      reg_barrier16(xx[0]);
      reg_barrier16(xx[1]);
      reg_barrier16(ll[0]);
      reg_barrier16(ll[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);  // every score of this buffer is in registers
      const uint32_t own0 = own;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sc[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) sc[x] = (hh[c][x] << 16) + (xx[c][x] << 8) + ll[c][x];  // mod 2^32: exact
        filter_chunk(sc, rbase + c * 16, r1, row_base, live, k, ext, thr, own, top);
      }
      if (own != own0) atomicMax(const_cast<uint32_t*>(&s_thr[lq]), own);
      if (gthr && own > pub && ((t & 31) == 31 || t == ntiles - 1)) {
        atomicMax(gthr, own);
        pub = own;
      }
    }
    // both halves of each query -> one list of k keys per (query, part)
    named_bar_sync(1, S_EPI_WARPS * 32);  // every tile consumed: the ring is free for the merge
    uint64_t* sk = reinterpret_cast<uint64_t*>(sRing);  // [SQ][S_KMAX], half 1's lists (32 KB of the ring)
    if (half == 1) {
#pragma unroll
      for (int i = 0; i < S_KMAX; ++i) sk[lq * S_KMAX + i] = top.v[i];
    }
    named_bar_sync(1, S_EPI_WARPS * 32);
    if (half == 0 && live) {
      uint64_t* dst = cand + ((int64_t)qg * n_parts + part) * k;
      const uint64_t* other = sk + lq * S_KMAX;
      int ib = 0;
      for (int i = 0; i < k; ++i) {
        const uint64_t bk = ib < S_KMAX ? other[ib] : 0;
        if (top.v[0] >= bk) {
          dst[i] = top.v[0];
#pragma unroll
          for (int j = 0; j < S_KMAX - 1; ++j) top.v[j] = top.v[j + 1];
          top.v[S_KMAX - 1] = 0;
        } else {
          dst[i] = bk;
          ++ib;
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

PFN_cuTensorMapEncodeTiled_v12000 search_encoder() {
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

cudaError_t map_bytes(CUtensorMap* m, const void* base, int64_t rows, int row_bytes, int box_rows) {
  auto enc = search_encoder();
  if (!enc) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)SKB, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

int g_search_sms[64];
bool g_search_attr[64];
bool g_search16_attr[64];
std::mutex g_search_mu;

}  // namespace

bool scan_exact_tc16_supported(int dim, int plane_bytes, int k) {
  return plane_bytes >= SKB && plane_bytes % 16 == 0 && (plane_bytes + SKB - 1) / SKB <= S16_MAX_QBOX &&
         dim <= plane_bytes && k >= 1 && k <= S_KMAX;
}

cudaError_t launch_scan_exact_tc16(const void* corpus_hi, const void* corpus_lo, int64_t count, int plane_bytes,
                                   const void* q_hi, const void* q_lo, int nq, int k, TcScanPlan plan,
                                   int64_t row_base, uint64_t* cand, uint32_t* qthr, uint32_t* err,
                                   cudaStream_t stream) {
  if (nq == 0 || count == 0) return cudaSuccess;
  const int nqb = (plane_bytes + SKB - 1) / SKB;
  if (nqb > S16_MAX_QBOX || plan.rows_per_part % SN16) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(corpus_hi) | reinterpret_cast<uintptr_t>(corpus_lo) |
       reinterpret_cast<uintptr_t>(q_hi) | reinterpret_cast<uintptr_t>(q_lo)) & 15)
    return cudaErrorMisalignedAddress;
  const int nst = 2;
  const int smem = 1024 + 2 * nqb * S_QBOX + nst * S16_STAGE + S_BAR_BYTES + S_THR_BYTES;
  if (smem > 232448 || nst * S16_STAGE < SQ * S_KMAX * 8) return cudaErrorInvalidValue;
  CUtensorMap mch, mcl, mqh, mql;
  cudaError_t e;
  if ((e = map_bytes(&mch, corpus_hi, count, plane_bytes, SN16)) != cudaSuccess) return e;
  if ((e = map_bytes(&mcl, corpus_lo, count, plane_bytes, SN16)) != cudaSuccess) return e;
  if ((e = map_bytes(&mqh, q_hi, nq, plane_bytes, SQ)) != cudaSuccess) return e;
  if ((e = map_bytes(&mql, q_lo, nq, plane_bytes, SQ)) != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(g_search_mu);
    if (dev >= 0 && dev < 64 && !g_search16_attr[dev]) {
      if ((e = cudaFuncSetAttribute(search_tc16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448)) !=
          cudaSuccess)
        return e;
      g_search16_attr[dev] = true;
    }
  }
  const int64_t grid = (int64_t)plan.n_parts * plan.n_qtiles;
  search_tc16_kernel<<<(unsigned)grid, S_THREADS, smem, stream>>>(mch, mcl, mqh, mql, count, nqb, nst, nq, k,
                                                                  plan.rows_per_part, plan.n_qtiles, plan.n_parts,
                                                                  row_base, cand, qthr, err);
  return cudaGetLastError();
}

// int16 rows (row_bytes apart) -> high-byte and low-byte planes of
// plane_bytes per row (zero padded): c = 256 * hi + lo, hi signed, lo unsigned.
__global__ void split_int16_kernel(const int16_t* __restrict__ src, int64_t rows, int dim, int src_row_bytes,
                                   int plane_bytes, uint8_t* __restrict__ hi, uint8_t* __restrict__ lo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one (row, 4-byte group of the planes)
  const int groups = plane_bytes / 4;
  if (i >= rows * groups) return;
  const int64_t r = i / groups;
  const int c0 = (int)(i % groups) * 4;
  const int16_t* row = reinterpret_cast<const int16_t*>(reinterpret_cast<const uint8_t*>(src) + r * src_row_bytes);
  uint32_t h = 0, l = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = c0 + j;
    const int v = c < dim ? (int)row[c] : 0;
    h |= (uint32_t)((v >> 8) & 0xff) << (8 * j);
    l |= (uint32_t)(v & 0xff) << (8 * j);
  }
  reinterpret_cast<uint32_t*>(hi + r * plane_bytes)[c0 / 4] = h;
  reinterpret_cast<uint32_t*>(lo + r * plane_bytes)[c0 / 4] = l;
}

cudaError_t launch_split_int16(const void* src, int64_t rows, int dim, int src_row_bytes, int plane_bytes, void* hi,
                               void* lo, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (plane_bytes % 16 || dim > plane_bytes || src_row_bytes < dim * 2) return cudaErrorInvalidValue;
  const int64_t n = rows * (plane_bytes / 4);
  split_int16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(static_cast<const int16_t*>(src), rows, dim,
                                                                      src_row_bytes, plane_bytes,
                                                                      static_cast<uint8_t*>(hi),
                                                                      static_cast<uint8_t*>(lo));
  return cudaGetLastError();
}

bool scan_exact_tc_supported(int elem, int row_bytes, int k, const void* corpus, const void* qcodes) {
  return elem == 1 && row_bytes >= SKB && (row_bytes + SKB - 1) / SKB <= S_MAX_QBOX && k >= 1 && k <= S_KMAX &&
         !(reinterpret_cast<uintptr_t>(corpus) & 15) && !(reinterpret_cast<uintptr_t>(qcodes) & 15) &&
         row_bytes % 16 == 0;
}

TcScanPlan plan_scan_exact_tc(int64_t count, int nq) {
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lk(g_search_mu);
    if (!g_search_sms[dev]) cudaDeviceGetAttribute(&g_search_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (g_search_sms[dev] > 0) sms = g_search_sms[dev];
  }
  TcScanPlan p;
  p.n_qtiles = (nq + SQ - 1) / SQ;
  // parts of at most 32768 rows (25 MB at D = 768: the query tiles reading a
  // part together keep it in L2)
  int64_t parts = (count + 32767) / 32768;
  // one CTA per SM: when the grid would be only a few waves, split the
  // corpus finer so that it fills whole waves
  const int64_t ctas = parts * p.n_qtiles;
  if (ctas < 4LL * sms) {
    const int64_t waves = (ctas + sms - 1) / sms;
    const int64_t want = waves * sms / p.n_qtiles;
    if (parts < want) parts = want;
  }
  int64_t rpp = (count + parts - 1) / parts;
  rpp = (rpp + SN - 1) / SN * SN;
  if (rpp < SN) rpp = SN;
  p.rows_per_part = rpp;
  p.n_parts = (int)((count + rpp - 1) / rpp);
  if (p.n_parts < 1) p.n_parts = 1;
  return p;
}

cudaError_t launch_scan_exact_tc(const void* corpus, int64_t count, int row_bytes, const void* qcodes, int nq, int k,
                                 TcScanPlan plan, int64_t row_base, uint64_t* cand, uint32_t* qthr, uint32_t* err,
                                 cudaStream_t stream) {
  if (nq == 0 || count == 0) return cudaSuccess;
  const int nqb = (row_bytes + SKB - 1) / SKB;
  if (nqb > S_MAX_QBOX) return cudaErrorInvalidValue;
  const int nst = nqb <= 6 ? 4 : 3;
  const int smem = 1024 + nqb * S_QBOX + nst * S_TILE + S_BAR_BYTES + S_THR_BYTES;
  if (smem > 232448) return cudaErrorInvalidValue;
  CUtensorMap mc, mq;
  cudaError_t e;
  if ((e = map_bytes(&mc, corpus, count, row_bytes, SN)) != cudaSuccess) return e;
  if ((e = map_bytes(&mq, qcodes, nq, row_bytes, SQ)) != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(g_search_mu);
    if (dev >= 0 && dev < 64 && !g_search_attr[dev]) {
      if ((e = cudaFuncSetAttribute(search_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448)) !=
          cudaSuccess)
        return e;
      g_search_attr[dev] = true;
    }
  }
  const int64_t grid = (int64_t)plan.n_parts * plan.n_qtiles;
  search_tc_kernel<<<(unsigned)grid, S_THREADS, smem, stream>>>(mc, mq, count, nqb, nst, nq, k, plan.rows_per_part,
                                                                plan.n_qtiles, plan.n_parts, row_base, cand, qthr,
                                                                err);
  return cudaGetLastError();
}

}  // namespace sem
