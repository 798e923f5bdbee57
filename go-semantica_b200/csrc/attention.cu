// Bidirectional GQA attention for EmbeddingGemma (runAttentionINT8 →
// MultiHeadAttentionChunked, internal/runtime/model_int8.go:455-500,
// internal/kernels/attention.go:178-310, softmax activation.go:161-213).
//
// The reference materialises the scores of every query row, takes the exact
// row max, applies its polynomial fastExp (which clamps arguments below -10 to
// zero) and multiplies by 1/sum. Because of that clamp an online-softmax
// rescale would change results, so this kernel makes two passes over the keys:
//   pass 1: fp16 scores on the tensor cores, only to find each row's max;
//   pass 2: scores with three-term fp16 products (hi*hi + hi*lo + lo*hi, where
//           x = hi + lo exactly to ~22 bits) for near-fp32 accuracy,
//           p = fastExp(score - max), row sums, and O += P V, again with
//           three-term products of split P and V.
// The max from pass 1 differs from the exact max by the fp16 error of one
// score; fastExp(x - d) = fastExp(x) * e^-d up to O(1e-3 d), and the common
// factor cancels in the normalisation.
//
// One CTA = 64 query rows of one (sequence, head); 8 warps. K/V tiles of 32
// keys are double-buffered with cp.async; all three query heads read the same
// single KV head (GQA), so K/V are shared in L2.
#include "common.cuh"
#include "kernels.h"

namespace sem {

namespace {
constexpr int HD = 256;           // head_dim
constexpr int QT = 64;            // query rows per CTA
constexpr int KT = 32;            // keys per tile
constexpr int LDH = HD + 8;       // padded smem row (halves): 528 bytes, conflict-free ldmatrix
constexpr int LDP = KT + 8;       // padded P row (halves): 80 bytes
constexpr int THREADS = 256;
constexpr int Q_HALVES = QT * LDH;
constexpr int KV_HALVES = KT * LDH;
constexpr int SMEM_BYTES = (2 * Q_HALVES + 2 * 4 * KV_HALVES + 2 * QT * LDP) * 2 + 4 * QT * 4;
}  // namespace

__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __half* __restrict__ qh, const __half* __restrict__ ql, const __half* __restrict__ kh,
                     const __half* __restrict__ kl, const __half* __restrict__ vh, const __half* __restrict__ vl,
                     int nh, float scale, SeqMeta meta, AttnTiles tiles, float* __restrict__ out,
                     uint32_t* __restrict__ absmax) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __half* sQh = reinterpret_cast<__half*>(smem_raw);
  __half* sQl = sQh + Q_HALVES;
  __half* sKV = sQl + Q_HALVES;  // [stage][4][KT][LDH]: Kh, Kl, Vh, Vl
  __half* sPh = sKV + 2 * 4 * KV_HALVES;
  __half* sPl = sPh + QT * LDP;
  float* sRed = reinterpret_cast<float*>(sPl + QT * LDP);  // [2][QT] maxima, then [2][QT] sums

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int tile = blockIdx.x, head = blockIdx.y;
  const int seq = tiles.tile_seq[tile];
  const int row0 = tiles.tile_row0[tile];
  const int s_beg = meta.cu_seqlens[seq], s_end = meta.cu_seqlens[seq + 1];
  const int n_rows = min(QT, s_end - row0);
  const int n_keys = s_end - s_beg;
  const int n_kt = (n_keys + KT - 1) / KT;

  // ---- load Q (hi, lo) ----
  for (int i = tid; i < QT * (HD / 8); i += THREADS) {
    int r = i / (HD / 8), c = i % (HD / 8);
    bool v = r < n_rows;
    int64_t src = ((int64_t)(v ? row0 + r : row0) * nh + head) * HD + c * 8;
    cp_async16(sQh + r * LDH + c * 8, qh + src, v);
    cp_async16(sQl + r * LDH + c * 8, ql + src, v);
  }
  cp_async_commit();

  auto load_kv = [&](int stage, int kt, bool with_lo_v) {
    __half* base = sKV + stage * 4 * KV_HALVES;
    const int nparts = with_lo_v ? 4 : 1;
    for (int i = tid; i < nparts * KT * (HD / 8); i += THREADS) {
      int part = i / (KT * (HD / 8));
      int rem = i % (KT * (HD / 8));
      int r = rem / (HD / 8), c = rem % (HD / 8);
      int key = kt * KT + r;
      bool v = key < n_keys;
      const __half* src = part == 0 ? kh : part == 1 ? kl : part == 2 ? vh : vl;
      cp_async16(base + part * KV_HALVES + r * LDH + c * 8, src + (int64_t)(s_beg + (v ? key : 0)) * HD + c * 8, v);
    }
  };

  const int r0 = 16 * (warp & 3);    // query rows of this warp (both passes)
  const int kk0 = 16 * (warp >> 2);  // key half of the tile for the score phase
  const int d0 = 128 * (warp >> 2);  // output dims for the PV phase

  // ================= pass 1: row maxima =================
  float mrun[2] = {-INFINITY, -INFINITY};
  load_kv(0, 0, false);
  cp_async_commit();
  for (int kt = 0; kt < n_kt; ++kt) {
    if (kt + 1 < n_kt) load_kv((kt + 1) & 1, kt + 1, false);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __half* sK = sKV + (kt & 1) * 4 * KV_HALVES;
    // four independent accumulator chains (k-step parity x key half) keep the
    // tensor pipe busy; they are summed once per tile
    float s4[2][2][4] = {};
#pragma unroll 4
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4], b[2][2];
      ldmatrix_x4(a[0], a[1], a[2], a[3], sQh + (r0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LDH + (2 * ks + (lane >> 4)) * 8);
      ldmatrix_x4(b[0][0], b[0][1], b[1][0], b[1][1],
                  sK + (kk0 + (lane & 7) + (lane >> 4) * 8) * LDH + (2 * ks + ((lane >> 3) & 1)) * 8);
      mma_f16(s4[ks & 1][0], a, b[0]);
      mma_f16(s4[ks & 1][1], a, b[1]);
    }
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = __fadd_rn(s4[0][nt][e], s4[1][nt][e]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int key = kt * KT + kk0 + nt * 8 + t4 * 2 + (e & 1);
        if (key < n_keys) mrun[e >> 1] = fmaxf(mrun[e >> 1], __fmul_rn(s[nt][e], scale));
      }
    __syncthreads();  // the buffer just read is refilled two iterations later
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrun[h] = fmaxf(mrun[h], __shfl_xor_sync(0xffffffffu, mrun[h], 1));
    mrun[h] = fmaxf(mrun[h], __shfl_xor_sync(0xffffffffu, mrun[h], 2));
  }
  if (t4 == 0) {
    sRed[(warp >> 2) * QT + r0 + g] = mrun[0];
    sRed[(warp >> 2) * QT + r0 + g + 8] = mrun[1];
  }
  __syncthreads();
  float mrow[2];
  mrow[0] = fmaxf(sRed[r0 + g], sRed[QT + r0 + g]);
  mrow[1] = fmaxf(sRed[r0 + g + 8], sRed[QT + r0 + g + 8]);

  // ================= pass 2: P, row sums, O = P V =================
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  float lsum[2] = {0.0f, 0.0f};

  load_kv(0, 0, true);
  cp_async_commit();
  for (int kt = 0; kt < n_kt; ++kt) {
    if (kt + 1 < n_kt) load_kv((kt + 1) & 1, kt + 1, true);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __half* sKh = sKV + (kt & 1) * 4 * KV_HALVES;
    const __half* sKl = sKh + KV_HALVES;
    const __half* sVh = sKl + KV_HALVES;
    const __half* sVl = sVh + KV_HALVES;
    // scores of rows r0..r0+15 x keys kk0..kk0+15
    // hi*hi and the two cross terms accumulate in separate chains, alternating
    // by k-step parity: eight independent MMA chains per warp instead of two
    float sm[2][2][4] = {}, sx[2][2][4] = {};
#pragma unroll 2
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t ah[4], al[4], bh[2][2], bl[2][2];
      const int qoff = (r0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LDH + (2 * ks + (lane >> 4)) * 8;
      const int koff = (kk0 + (lane & 7) + (lane >> 4) * 8) * LDH + (2 * ks + ((lane >> 3) & 1)) * 8;
      ldmatrix_x4(ah[0], ah[1], ah[2], ah[3], sQh + qoff);
      ldmatrix_x4(al[0], al[1], al[2], al[3], sQl + qoff);
      ldmatrix_x4(bh[0][0], bh[0][1], bh[1][0], bh[1][1], sKh + koff);
      ldmatrix_x4(bl[0][0], bl[0][1], bl[1][0], bl[1][1], sKl + koff);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        mma_f16(sx[ks & 1][nt], al, bh[nt]);
        mma_f16(sx[ks & 1][nt], ah, bl[nt]);
        mma_f16(sm[ks & 1][nt], ah, bh[nt]);
      }
    }
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        s[nt][e] = __fadd_rn(__fadd_rn(sm[0][nt][e], sm[1][nt][e]), __fadd_rn(sx[0][nt][e], sx[1][nt][e]));
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int key = kt * KT + kk0 + nt * 8 + t4 * 2 + (e & 1);
        float sc = __fmul_rn(s[nt][e], scale);  // score *= scale (attention.go:300)
        p[e] = key < n_keys ? fast_exp_ref(__fsub_rn(sc, mrow[e >> 1])) : 0.0f;
        lsum[e >> 1] = __fadd_rn(lsum[e >> 1], p[e]);
      }
      __half h0, l0, h1, l1;
      const int col = kk0 + nt * 8 + t4 * 2;
      split_half(p[0], h0, l0);
      split_half(p[1], h1, l1);
      *reinterpret_cast<__half2*>(sPh + (r0 + g) * LDP + col) = __halves2half2(h0, h1);
      *reinterpret_cast<__half2*>(sPl + (r0 + g) * LDP + col) = __halves2half2(l0, l1);
      split_half(p[2], h0, l0);
      split_half(p[3], h1, l1);
      *reinterpret_cast<__half2*>(sPh + (r0 + g + 8) * LDP + col) = __halves2half2(h0, h1);
      *reinterpret_cast<__half2*>(sPl + (r0 + g + 8) * LDP + col) = __halves2half2(l0, l1);
    }
    __syncthreads();
    // O[r0..r0+15][d0..d0+127] += P[r0.., 0..31] V[0..31][d0..]
#pragma unroll
    for (int kstep = 0; kstep < KT / 16; ++kstep) {
      uint32_t ph[4], pl[4];
      const int poff = (r0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LDP + (2 * kstep + (lane >> 4)) * 8;
      ldmatrix_x4(ph[0], ph[1], ph[2], ph[3], sPh + poff);
      ldmatrix_x4(pl[0], pl[1], pl[2], pl[3], sPl + poff);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t vhf[2][2], vlf[2][2];
        const int voff = (16 * kstep + (lane & 7) + ((lane >> 3) & 1) * 8) * LDH + ((d0 + 16 * dp) / 8 + (lane >> 4)) * 8;
        ldmatrix_x4_trans(vhf[0][0], vhf[0][1], vhf[1][0], vhf[1][1], sVh + voff);
        ldmatrix_x4_trans(vlf[0][0], vlf[0][1], vlf[1][0], vlf[1][1], sVl + voff);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mma_f16(o[2 * dp + j], pl, vhf[j]);
          mma_f16(o[2 * dp + j], ph, vlf[j]);
          mma_f16(o[2 * dp + j], ph, vhf[j]);
        }
      }
    }
    __syncthreads();  // P and this K/V buffer are rewritten next
  }

  // ---- row sums over both key halves, normalise, store, absmax ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lsum[h] = __fadd_rn(lsum[h], __shfl_xor_sync(0xffffffffu, lsum[h], 1));
    lsum[h] = __fadd_rn(lsum[h], __shfl_xor_sync(0xffffffffu, lsum[h], 2));
  }
  float* sSum = sRed + 2 * QT;
  if (t4 == 0) {
    sSum[(warp >> 2) * QT + r0 + g] = lsum[0];
    sSum[(warp >> 2) * QT + r0 + g + 8] = lsum[1];
  }
  __syncthreads();
  float inv[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float l = __fadd_rn(sSum[r0 + g + 8 * h], sSum[QT + r0 + g + 8 * h]);
    inv[h] = l > 0.0f ? __fdiv_rn(1.0f, l) : 0.0f;  // l >= fastExp(~0) ~ 1 for every valid row
  }
  float amax = 0.0f;
  const int ld = nh * HD;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + g + 8 * h;
    const bool valid = r < n_rows;
    float* dst = out + (int64_t)(row0 + (valid ? r : 0)) * ld + head * HD + d0 + t4 * 2;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      float v0 = __fmul_rn(o[nt][2 * h], inv[h]);
      float v1 = __fmul_rn(o[nt][2 * h + 1], inv[h]);
      if (valid) {
        *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(v0, v1);
        amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
      }
    }
  }
  amax = warp_max(amax);
  if (lane == 0 && absmax) atomicMax(&absmax[seq], __float_as_uint(amax));
}

cudaError_t launch_attention(const __half* qh, const __half* ql, const __half* kh, const __half* kl, const __half* vh,
                             const __half* vl, int num_heads, float scale, SeqMeta meta, AttnTiles tiles, float* out,
                             uint32_t* absmax, cudaStream_t stream) {
  if (tiles.n_tiles == 0) return cudaSuccess;
  cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  dim3 grid(tiles.n_tiles, num_heads);
  attention_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(qh, ql, kh, kl, vh, vl, num_heads, scale, meta, tiles, out,
                                                         absmax);
  return cudaGetLastError();
}

}  // namespace sem
