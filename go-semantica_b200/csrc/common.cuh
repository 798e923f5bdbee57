// Shared device helpers for the sm_100a kernels.
//
// Every kernel source is compiled with --fmad=false: the reference computes in
// unfused float32 except where its amd64 assembly uses VFMADD231PS, and those
// places call fmaf() explicitly here. Keeping contraction off is what makes the
// element-wise kernels bit-identical to the reference's Go code.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sem {

constexpr float kFloatMagic = 12582912.0f;      // 1.5 * 2^23
constexpr int kFloatMagicBits = 0x4B400000;     // bit pattern of kFloatMagic

// fastExp (internal/kernels/activation.go:100-145), restated operation by
// operation and without branches: every case is computed and selected, and
// the truncation int32(y) is taken as trunc(y), whose integer value is read
// out of the float with a 1.5 * 2^23 add (no float<->int conversion
// instructions). The results are those of the reference's branchy code.
__device__ __forceinline__ float fast_exp_ref(float x) {
  const float y = __fmul_rn(x, 1.442695041f);
  const float yt = truncf(y);  // == (float)int32(y), truncation toward zero
  const int ip = __float_as_int(__fadd_rn(yt, 12582912.0f)) - 0x4B400000;
  const float f = __fsub_rn(y, yt);
  const float c1 = 0.693147180559945f, c2 = 0.240226506959101f, c3 = 0.055504108664821f,
              c4 = 0.009676036358193f;
  const float poly = __fadd_rn(
      1.0f, __fmul_rn(f, __fadd_rn(c1, __fmul_rn(f, __fadd_rn(c2, __fmul_rn(f, __fadd_rn(c3, __fmul_rn(f, c4))))))));
  float r = __fmul_rn(poly, __uint_as_float((uint32_t)(ip + 127) << 23));
  r = ip < -126 ? 0.0f : r;
  r = ip > 127 ? 3.402823e+38f : r;
  r = x > 10.0f ? 22026.4657948f : r;
  return x < -10.0f ? 0.0f : r;
}

// fast_exp_ref for x <= 0: from -10 up the exponent int32(x * log2e) lies in
// [-14, 0], so of the four clamps only x < -10 can act and the result is
// fast_exp_ref's bit for bit (for a NaN argument it is NaN where fast_exp_ref
// gives its overflow value; the one caller's result is NaN either way).
__device__ __forceinline__ float fast_exp_nonpos(float x) {
  const float y = __fmul_rn(x, 1.442695041f);
  const float yt = truncf(y);
  const int ip = __float_as_int(__fadd_rn(yt, 12582912.0f)) - 0x4B400000;
  const float f = __fsub_rn(y, yt);
  const float c1 = 0.693147180559945f, c2 = 0.240226506959101f, c3 = 0.055504108664821f,
              c4 = 0.009676036358193f;
  const float poly = __fadd_rn(
      1.0f, __fmul_rn(f, __fadd_rn(c1, __fmul_rn(f, __fadd_rn(c2, __fmul_rn(f, __fadd_rn(c3, __fmul_rn(f, c4))))))));
  const float r = __fmul_rn(poly, __uint_as_float((uint32_t)(ip + 127) << 23));
  return x < -10.0f ? 0.0f : r;
}

// GELUQuickSIMD element (activation.go:47-95): x * sigmoid(1.702 x) through
// fastExp. Both of the reference's branches evaluate fastExp(-|1.702 x|) and
// divide by 1 + e; only the numerator differs (1, or e for negative x).
__device__ __forceinline__ float gelu_quick_ref(float x) {
  const float sx = __fmul_rn(1.702f, x);
  const float e = fast_exp_nonpos(-fabsf(sx));
  const float sig = __fdiv_rn(sx >= 0.0f ? 1.0f : e, __fadd_rn(1.0f, e));
  return __fmul_rn(x, sig);
}

// Sum of squares of a row in the order of dotProductAVX2Asm
// (internal/kernels/simd_amd64.s:19-76): 8 fused lane accumulators over the row
// (lane l takes elements 8v+l), then the VEXTRACTF128/VADDPS/VHADDPS horizontal
// sum. Computed by the 8 consecutive lanes of a warp that share `sub` = lane & 7;
// every lane of the group receives the total. n must be a multiple of 8.
__device__ __forceinline__ float row_sumsq_ref(const float* __restrict__ x, int n, int sub) {
  float acc = 0.0f;
#pragma unroll 8
  for (int v = 0; v < n / 8; ++v) {
    float t = x[8 * v + sub];
    acc = fmaf(t, t, acc);
  }
  const unsigned full = 0xffffffffu;
  float hi = __shfl_down_sync(full, acc, 4, 8);   // sub 0..3 receive acc[sub+4]
  float s = __fadd_rn(acc, hi);                   // s_i = acc_i + acc_{i+4}
  float s1 = __shfl_down_sync(full, s, 1, 8);
  float p = __fadd_rn(s, s1);                     // sub0: s0+s1, sub2: s2+s3
  float p2 = __shfl_down_sync(full, p, 2, 8);
  float tot = __fadd_rn(p, p2);                   // sub0: (s0+s1)+(s2+s3)
  return __shfl_sync(full, tot, 0, 8);
}

// RMSNorm inverse scale (internal/kernels/norm.go:8-36):
// 1 / float32(sqrt(float64(sumSq/n + eps))). Rounding a square root first to
// float64 and then to float32 gives the correctly rounded float32 root (53 >=
// 2 * 24 + 2 bits makes the double rounding innocuous; also checked on every
// non-negative float), so the IEEE float32 square root computes it; 1 / rms
// is the IEEE reciprocal.
__device__ __forceinline__ float rms_inv_ref(float sumsq, int n, float eps) {
  float mean = __fdiv_rn(sumsq, (float)n);
  float rms = __fsqrt_rn(__fadd_rn(mean, eps));
  return __frcp_rn(rms);
}

// Per-sequence activation scale (quantize.go:60-61) from an absmax bit pattern.
__device__ __forceinline__ void seq_scale_ref(uint32_t absmax_bits, float* scale, float* inv) {
  float m = __uint_as_float(absmax_bits);
  if (m == 0.0f) {
    *scale = 1.0f;
    *inv = 0.0f;  // every code is 0 (quantize.go:50-58)
    return;
  }
  float s = __fdiv_rn(m, 127.0f);
  *scale = s;
  *inv = __fdiv_rn(1.0f, s);
}

// quantizeInto element (quantize.go:92-103): round half away from zero of the
// exact float64 product x * inv, clamped to [-127, 127], computed in float32
// only (float64 is slow on the GPU). The exact product x * inv equals
// p + e with p = fl(x * inv) and e = fma(x, inv, -p) (exact). With t = trunc(p),
// p - t is exact; unless |p - t| is exactly one half, |e| (at most half an ulp
// of p) cannot move the product across the half, and at exactly one half the
// sign of e decides. Returns the integer code as a float.
__device__ __forceinline__ float quant_code_f32(float x, float inv) {
  const float p = __fmul_rn(x, inv);
  const float e = __fmaf_rn(x, inv, -p);
  const float t = truncf(p);
  const float ad = fabsf(__fsub_rn(p, t));
  const bool pos = p > 0.0f;
  const bool away = ad > 0.5f || (ad == 0.5f && (pos ? e >= 0.0f : e <= 0.0f));
  const float n = away ? (pos ? __fadd_rn(t, 1.0f) : __fsub_rn(t, 1.0f)) : t;
  return fminf(fmaxf(n, -127.0f), 127.0f);
}

// Four codes of quantizeInto as packed fp16. Rounding preserves order and
// every half-integer of magnitude below 2^23 is a float, so round-half-away of
// the exact product equals rint(p) of the rounded product p unless p itself is
// a half-integer; only then (rarely) does the exact path above run. Larger
// |p| clamp to +-127 on both paths, NaN to -127 on both.
__device__ __forceinline__ uint2 quant_codes4(float4 x, float inv) {
  const float e[4] = {x.x, x.y, x.z, x.w};
  float n[4];
  bool tie = false;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float p = __fmul_rn(e[k], inv);
    n[k] = rintf(p);
    tie |= fabsf(__fsub_rn(p, n[k])) == 0.5f;
    n[k] = fminf(fmaxf(n[k], -127.0f), 127.0f);
  }
  if (tie) {
#pragma unroll
    for (int k = 0; k < 4; ++k) n[k] = quant_code_f32(e[k], inv);
  }
  __half2 h[2] = {__floats2half2_rn(n[0], n[1]), __floats2half2_rn(n[2], n[3])};
  return *reinterpret_cast<uint2*>(h);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  uint32_t s = smem_u32(smem);
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Packed fp32 pair arithmetic (sm_100+).
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
  a = __uint_as_float((uint32_t)v);
  b = __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// fastExp of a pair with packed fp32 arithmetic, fast_exp_ref's operations on
// each element. ptxas contracts a packed multiply with the add consuming it
// into one fused multiply-add (even with .rn), so about one result in ten
// differs from fast_exp_ref by an ulp: used only where tensor-core sums
// already set the precision (the attention softmax), never where a result
// must be bit-exact. For |x| <= 10 the exponent int32(x * log2e) lies in
// [-15, 15], so only the two argument clamps remain.
__device__ __forceinline__ uint64_t fast_exp_ref2(uint64_t x2) {
  const uint64_t y2 = mul2(x2, pack2(1.442695041f, 1.442695041f));
  float y0, y1;
  unpack2(y2, y0, y1);
  const uint64_t yt2 = pack2(truncf(y0), truncf(y1));
  float m0, m1;
  unpack2(add2(yt2, pack2(12582912.0f, 12582912.0f)), m0, m1);
  const int ip0 = __float_as_int(m0) - 0x4B400000, ip1 = __float_as_int(m1) - 0x4B400000;
  const uint64_t f2 = sub2(y2, yt2);
  uint64_t t = mul2(f2, pack2(0.009676036358193f, 0.009676036358193f));
  t = add2(pack2(0.055504108664821f, 0.055504108664821f), t);
  t = mul2(f2, t);
  t = add2(pack2(0.240226506959101f, 0.240226506959101f), t);
  t = mul2(f2, t);
  t = add2(pack2(0.693147180559945f, 0.693147180559945f), t);
  t = mul2(f2, t);
  t = add2(pack2(1.0f, 1.0f), t);
  float r0, r1;
  unpack2(mul2(t, pack2(__uint_as_float((uint32_t)(ip0 + 127) << 23), __uint_as_float((uint32_t)(ip1 + 127) << 23))),
          r0, r1);
  float x0, x1;
  unpack2(x2, x0, x1);
  r0 = x0 > 10.0f ? 22026.4657948f : (x0 < -10.0f ? 0.0f : r0);
  r1 = x1 > 10.0f ? 22026.4657948f : (x1 < -10.0f ? 0.0f : r1);
  return pack2(r0, r1);
}

// Splits x into hi + lo halves (hi = fp16(x), lo = fp16(x - hi)) for the
// three-term fp16 products that give near-fp32 accuracy on the tensor cores.
__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}

}  // namespace sem
