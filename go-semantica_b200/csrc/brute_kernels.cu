// search/brute scan + top-k (Index.searchNormalized, search/brute/index.go:55-154).
//
// Two scoring contracts:
//  * exact (the integer contract): the query is quantised like the stored
//    rows (quant.go:17-41) and score = sum int32(q) * int32(v), accumulated
//    exactly (dp4a for int8, IMAD for int16);
//  * float (the reference's own arithmetic): score = sum q_f32 * (code * 1/127)
//    with the 8 lane accumulators of dotInt8AVX2 / dotInt16AVX2 / dotFloat32AVX2
//    (dot_amd64.s) and the 4-way LUT tail of quant.go:83-135, bit for bit.
// Top-k uses a total order: score descending, then row ascending. Candidates
// are 64-bit keys (order-preserving score bits << 32 | ~row) so "larger key is
// better" and ties resolve to the lower row.
//
// Layout: rows are stored padded to a 16-byte multiple (zero codes add
// nothing). One CTA = 8 queries (one per warp) x a contiguous row chunk,
// streamed through shared memory in double-buffered tiles of 32 rows (16 for
// float32 storage); lane i scores row i of each tile and keeps a private
// sorted top-K in registers; the warp then merges its 32 lists.
#include "common.cuh"
#include "kernels.h"

namespace sem {

namespace {
constexpr int QB = 8;        // queries per CTA
constexpr int THREADS = 256; // 8 warps

__device__ __forceinline__ uint64_t key_from_int(int32_t score, uint32_t row) {
  return ((uint64_t)((uint32_t)score ^ 0x80000000u) << 32) | (uint64_t)(0xffffffffu - row);
}
__device__ __forceinline__ uint64_t key_from_float(float score, uint32_t row) {
  uint32_t b = __float_as_uint(score);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xffffffffu - row);
}
__device__ __forceinline__ float float_from_key(uint64_t key) {
  uint32_t b = (uint32_t)(key >> 32);
  b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
  return __uint_as_float(b);
}

template <int K>
struct TopK {
  uint64_t v[K];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] = 0;
  }
  __device__ __forceinline__ void push(uint64_t key) {
    if (key <= v[K - 1]) return;
    v[K - 1] = key;
#pragma unroll
    for (int i = K - 1; i > 0; --i) {
      if (v[i] > v[i - 1]) {
        uint64_t t = v[i]; v[i] = v[i - 1]; v[i - 1] = t;
      }
    }
  }
  __device__ __forceinline__ void pop() {
#pragma unroll
    for (int i = 0; i < K - 1; ++i) v[i] = v[i + 1];
    v[K - 1] = 0;
  }
};

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t y = __shfl_xor_sync(0xffffffffu, x, o);
    x = y > x ? y : x;
  }
  return x;
}

// Warp merge of 32 sorted lists: emits the best `k` keys in order to dst.
template <int K>
__device__ __forceinline__ void warp_emit(TopK<K>& t, int k, uint64_t* dst) {
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < k; ++i) {
    uint64_t best = warp_max_u64(t.v[0]);
    if (lane == 0) dst[i] = best;
    // keys are unique (row bits differ), so exactly one lane owns `best`
    if (best != 0 && t.v[0] == best) t.pop();
  }
}

// ---- per-element dot helpers over a 16-byte chunk ----
__device__ __forceinline__ int dot16_i8(const uint4& a, const uint4& b, int acc) {
  acc = __dp4a((int)a.x, (int)b.x, acc);
  acc = __dp4a((int)a.y, (int)b.y, acc);
  acc = __dp4a((int)a.z, (int)b.z, acc);
  acc = __dp4a((int)a.w, (int)b.w, acc);
  return acc;
}
__device__ __forceinline__ int dot_word_i16(uint32_t a, uint32_t b, int acc) {
  acc += (int)(int16_t)(a & 0xffff) * (int)(int16_t)(b & 0xffff);
  acc += ((int)a >> 16) * ((int)b >> 16);
  return acc;
}
__device__ __forceinline__ int dot16_i16(const uint4& a, const uint4& b, int acc) {
  acc = dot_word_i16(a.x, b.x, acc);
  acc = dot_word_i16(a.y, b.y, acc);
  acc = dot_word_i16(a.z, b.z, acc);
  acc = dot_word_i16(a.w, b.w, acc);
  return acc;
}

constexpr float kInv127 = 0.0078740157f;      // dot_amd64.s:5
constexpr float kInv32767 = 0.000030518509f;  // dot_amd64.s:8

// Reference float dot of one stored row (smem) with a float query (smem).
// ELEM 1: dotInt8 (quant.go:83-108); 2: dotInt16 (:110-135); 4: dotFloat32 (index.go:198-214).
template <int ELEM>
__device__ float ref_float_dot(const uint8_t* row, const float* q, int dim) {
  float sum = 0.0f;
  int start = 0;
  if (dim >= 8) {
    const int n = dim & ~7;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < n; b += 8) {
#pragma unroll
      for (int l = 0; l < 8; ++l) {
        if (ELEM == 4) {
          float v = reinterpret_cast<const float*>(row)[b + l];
          acc[l] = fmaf(q[b + l], v, acc[l]);  // VFMADD231PS
        } else {
          float c = ELEM == 1 ? (float)reinterpret_cast<const int8_t*>(row)[b + l]
                              : (float)reinterpret_cast<const int16_t*>(row)[b + l];
          float t = __fmul_rn(c, ELEM == 1 ? kInv127 : kInv32767);
          t = __fmul_rn(t, q[b + l]);
          acc[l] = __fadd_rn(acc[l], t);
        }
      }
    }
    float s0 = __fadd_rn(acc[0], acc[4]), s1 = __fadd_rn(acc[1], acc[5]);
    float s2 = __fadd_rn(acc[2], acc[6]), s3 = __fadd_rn(acc[3], acc[7]);
    sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)));
    start = n;
  }
  if (ELEM == 4) {
    for (int i = start; i < dim; ++i)
      sum = __fadd_rn(sum, __fmul_rn(reinterpret_cast<const float*>(row)[i], q[i]));
    return sum;
  }
  auto lut = [&](int i) -> float {
    int c = ELEM == 1 ? (int)reinterpret_cast<const int8_t*>(row)[i] : (int)reinterpret_cast<const int16_t*>(row)[i];
    const int lim = ELEM == 1 ? 127 : 32767;
    if (c < -lim) c = -lim;
    return __fmul_rn((float)c, ELEM == 1 ? kInv127 : kInv32767);
  };
  float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  int i = start;
  for (; i + 4 <= dim; i += 4) {
    a0 = __fadd_rn(a0, __fmul_rn(q[i], lut(i)));
    a1 = __fadd_rn(a1, __fmul_rn(q[i + 1], lut(i + 1)));
    a2 = __fadd_rn(a2, __fmul_rn(q[i + 2], lut(i + 2)));
    a3 = __fadd_rn(a3, __fmul_rn(q[i + 3], lut(i + 3)));
  }
  sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3));
  for (; i < dim; ++i) sum = __fadd_rn(sum, __fmul_rn(q[i], lut(i)));
  return sum;
}
}  // namespace

// MODE 0: exact integer scores, MODE 1: reference float scores.
template <int MODE, int ELEM, int TR, int KMAX>
__global__ void __launch_bounds__(THREADS)
    scan_kernel(const uint8_t* __restrict__ corpus, int64_t count, int dim, int row_bytes,
                const uint8_t* __restrict__ queries, int nq, int k, int64_t rows_per_chunk, int64_t row_base,
                uint64_t* __restrict__ cand) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int ld = row_bytes + 16;  // padded smem row: conflict-free 16-byte reads
  uint8_t* tiles = smem;
  uint8_t* sq = smem + 2 * TR * ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qbase = blockIdx.y * QB;
  const int qrow_bytes = MODE == 0 ? row_bytes : dim * 4;

  // queries of this CTA (zero rows past nq)
  for (int i = tid; i < QB * (qrow_bytes / 4); i += THREADS) {
    int qi = i / (qrow_bytes / 4), w = i % (qrow_bytes / 4);
    uint32_t v = 0;
    if (qbase + qi < nq) v = reinterpret_cast<const uint32_t*>(queries + (int64_t)(qbase + qi) * qrow_bytes)[w];
    reinterpret_cast<uint32_t*>(sq + qi * qrow_bytes)[w] = v;
  }

  const int64_t r_beg = (int64_t)blockIdx.x * rows_per_chunk;
  const int64_t r_end = min(count, r_beg + rows_per_chunk);
  const int64_t ntiles = r_beg < r_end ? (r_end - r_beg + TR - 1) / TR : 0;
  const int chunks16 = row_bytes / 16;

  auto load_tile = [&](int buf, int64_t t) {
    uint8_t* dst = tiles + buf * TR * ld;
    for (int i = tid; i < TR * chunks16; i += THREADS) {
      int r = i / chunks16, c = i % chunks16;
      int64_t row = r_beg + t * TR + r;
      bool v = row < r_end;
      cp_async16(dst + r * ld + c * 16, corpus + (v ? row : 0) * (int64_t)row_bytes + c * 16, v);
    }
  };

  TopK<KMAX> top;
  top.init();
  if (ntiles > 0) load_tile(0, 0);
  cp_async_commit();
  for (int64_t t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) load_tile((t + 1) & 1, t + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* tb = tiles + (t & 1) * TR * ld;
    for (int r = lane; r < TR; r += 32) {
      int64_t row = r_beg + t * TR + r;
      if (row >= r_end) break;
      const uint8_t* rp = tb + r * ld;
      uint64_t key;
      if (MODE == 0) {
        const uint8_t* qp = sq + warp * row_bytes;
        int acc = 0;
        for (int c = 0; c < chunks16; ++c) {
          uint4 a = *reinterpret_cast<const uint4*>(rp + c * 16);
          uint4 b = *reinterpret_cast<const uint4*>(qp + c * 16);
          acc = ELEM == 1 ? dot16_i8(a, b, acc) : dot16_i16(a, b, acc);
        }
        key = key_from_int(acc, (uint32_t)(row_base + row));
      } else {
        const float* qp = reinterpret_cast<const float*>(sq + warp * qrow_bytes);
        key = key_from_float(ref_float_dot<ELEM>(rp, qp, dim), (uint32_t)(row_base + row));
      }
      top.push(key);
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  const int q = qbase + warp;
  if (q < nq) warp_emit<KMAX>(top, k, cand + ((int64_t)q * gridDim.x + blockIdx.x) * k);
}

// Final merge: one warp per query over `lists` lists of k candidate keys;
// list j of query q starts at cand + q * q_stride + j * list_stride.
template <int KMAX>
__global__ void topk_merge_kernel(const uint64_t* __restrict__ cand, int lists, int64_t list_stride,
                                  int64_t q_stride, int nq, int k, int k_out,
                                  bool float_keys, int elem, int32_t* __restrict__ out_rows,
                                  int32_t* __restrict__ out_scores, float* __restrict__ out_dist,
                                  uint64_t* __restrict__ out_keys) {
  __shared__ uint64_t s_keys[THREADS / 32][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x * (THREADS / 32) + warp;
  if (q >= nq) return;  // whole warp exits together
  TopK<KMAX> top;
  top.init();
  const uint64_t* src = cand + (int64_t)q * q_stride;
  for (int64_t i = lane; i < (int64_t)lists * k; i += 32) top.push(src[(i / k) * list_stride + i % k]);
  uint64_t* keys = s_keys[warp];
  warp_emit<KMAX>(top, k_out, keys);
  __syncwarp();
  const double sc2 = elem == 1 ? 127.0 * 127.0 : 32767.0 * 32767.0;
  for (int i = lane; i < k_out; i += 32) {
    uint64_t key = keys[i];
    int64_t o = (int64_t)q * k_out + i;
    if (out_keys) out_keys[o] = key;
    bool empty = key == 0;
    uint32_t row = 0xffffffffu - (uint32_t)key;
    if (out_rows) out_rows[o] = empty ? -1 : (int32_t)row;
    if (float_keys) {
      float d = empty ? 0.0f : float_from_key(key);
      if (out_dist) out_dist[o] = d;
      if (out_scores) out_scores[o] = 0;
    } else {
      int32_t s = empty ? 0 : (int32_t)((uint32_t)(key >> 32) ^ 0x80000000u);
      if (out_scores) out_scores[o] = s;
      if (out_dist) out_dist[o] = empty ? 0.0f : (float)((double)s / sc2);
    }
  }
}

namespace {
template <int MODE, int ELEM, int TR, int KMAX>
cudaError_t launch_scan_t(const void* corpus, int64_t count, int dim, const void* q, int nq, int k, ScanPlan plan,
                          uint64_t* cand, cudaStream_t stream) {
  int row_bytes = ((dim * ELEM + 15) / 16) * 16;
  int qrow_bytes = MODE == 0 ? row_bytes : dim * 4;
  size_t smem = (size_t)2 * TR * (row_bytes + 16) + (size_t)QB * qrow_bytes;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  auto kern = scan_kernel<MODE, ELEM, TR, KMAX>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(plan.chunks, (nq + QB - 1) / QB);
  kern<<<grid, THREADS, smem, stream>>>(static_cast<const uint8_t*>(corpus), count, dim, row_bytes,
                                        static_cast<const uint8_t*>(q), nq, k, plan.rows_per_chunk, plan.row_base,
                                        cand);
  return cudaGetLastError();
}

template <int MODE, int ELEM, int TR>
cudaError_t dispatch_k(const void* corpus, int64_t count, int dim, const void* q, int nq, int k, ScanPlan plan,
                       uint64_t* cand, cudaStream_t stream) {
  if (k <= 16) return launch_scan_t<MODE, ELEM, TR, 16>(corpus, count, dim, q, nq, k, plan, cand, stream);
  if (k <= 64) return launch_scan_t<MODE, ELEM, TR, 64>(corpus, count, dim, q, nq, k, plan, cand, stream);
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_scan_exact(const void* corpus, int elem, int64_t count, int dim, const void* qcodes, int nq, int k,
                              ScanPlan plan, uint64_t* cand, cudaStream_t stream) {
  if (nq == 0 || plan.chunks == 0) return cudaSuccess;
  if (elem == 1) return dispatch_k<0, 1, 32>(corpus, count, dim, qcodes, nq, k, plan, cand, stream);
  if (elem == 2) return dispatch_k<0, 2, 32>(corpus, count, dim, qcodes, nq, k, plan, cand, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_scan_float(const void* corpus, int elem, int64_t count, int dim, const float* queries, int nq,
                              int k, ScanPlan plan, uint64_t* cand, cudaStream_t stream) {
  if (nq == 0 || plan.chunks == 0) return cudaSuccess;
  if (elem == 1) return dispatch_k<1, 1, 32>(corpus, count, dim, queries, nq, k, plan, cand, stream);
  if (elem == 2) return dispatch_k<1, 2, 32>(corpus, count, dim, queries, nq, k, plan, cand, stream);
  if (elem == 4) return dispatch_k<1, 4, 16>(corpus, count, dim, queries, nq, k, plan, cand, stream);
  return cudaErrorInvalidValue;
}

// normalize (builder.go:129-141) then quantizeInt8/16 (quant.go:17-41) or a
// float copy, one thread per row so the float64 sum runs in the reference's
// sequential order. out rows are out_row_bytes apart (zero padded).
__global__ void normalize_quantize_kernel(const float* __restrict__ in, int64_t count, int dim, int quant,
                                          int out_row_bytes, bool normalize, uint8_t* __restrict__ out) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= count) return;
  const float* v = in + r * dim;
  float norm = 1.0f;
  bool scale = false;
  if (normalize) {
    double sum = 0.0;
    for (int i = 0; i < dim; ++i) sum += (double)__fmul_rn(v[i], v[i]);
    if (sum != 0.0) {
      norm = (float)(1.0 / sqrt(sum));
      scale = true;
    }
  }
  uint8_t* o = out + r * (int64_t)out_row_bytes;
  for (int i = 0; i < dim; ++i) {
    float x = scale ? __fmul_rn(v[i], norm) : v[i];
    if (quant == 0) {
      reinterpret_cast<float*>(o)[i] = x;
      continue;
    }
    if (x > 1.0f) x = 1.0f;
    else if (x < -1.0f) x = -1.0f;
    if (quant == 1) reinterpret_cast<int8_t*>(o)[i] = (int8_t)(int)round((double)x * 127.0);
    else reinterpret_cast<int16_t*>(o)[i] = (int16_t)(int)round((double)x * 32767.0);
  }
  const int elem = quant == 0 ? 4 : quant;
  for (int b = dim * elem; b < out_row_bytes; ++b) o[b] = 0;
}

cudaError_t launch_normalize_quantize(const float* in, int64_t count, int dim, int quant, int out_row_bytes,
                                      bool normalize, void* out, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  normalize_quantize_kernel<<<(unsigned)((count + 127) / 128), 128, 0, stream>>>(
      in, count, dim, quant, out_row_bytes, normalize, static_cast<uint8_t*>(out));
  return cudaGetLastError();
}

cudaError_t launch_topk_merge(const uint64_t* cand, int lists, int64_t list_stride, int64_t q_stride, int nq, int k,
                              int k_out, bool float_keys, int elem, int32_t* out_rows, int32_t* out_scores,
                              float* out_dist, uint64_t* out_keys, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  if (k_out > 64 || k_out > k) return cudaErrorInvalidValue;
  unsigned blocks = (unsigned)((nq + THREADS / 32 - 1) / (THREADS / 32));
  if (k_out <= 16)
    topk_merge_kernel<16><<<blocks, THREADS, 0, stream>>>(cand, lists, list_stride, q_stride, nq, k, k_out, float_keys,
                                                           elem, out_rows, out_scores, out_dist, out_keys);
  else
    topk_merge_kernel<64><<<blocks, THREADS, 0, stream>>>(cand, lists, list_stride, q_stride, nq, k, k_out, float_keys,
                                                           elem, out_rows, out_scores, out_dist, out_keys);
  return cudaGetLastError();
}

}  // namespace sem
