/*
 * semantica_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of go-semantica's INT8 embedding forward pass
 * (internal/runtime, internal/kernels, internal/gguf) and of search/brute.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * it, as the checker; the product library never links or calls it.
 *
 * Floating-point order: the reference runs on amd64 with AVX2 / AVX512-VNNI
 * assembly. Where that assembly fixes an accumulation order (8-lane FMA
 * accumulators followed by a horizontal add) this file reproduces that lane
 * order with explicit fmaf(); everywhere else operations are plain, unfused
 * float32 (the file is compiled with -ffp-contract=off, matching Go's default
 * amd64 code generation, which does not fuse multiply-adds).
 *
 * Parity status: partially pinned (see semantica_oracle.h).
 */
#define _GNU_SOURCE
#include "semantica_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static void seterr(char *err, int errlen, const char *fmt, ...) {
    if (!err || errlen <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
}

static inline float bits_to_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }

/* Which build of the reference to follow. The reference selects its kernels at
 * build and run time: 0 = amd64 on an AVX512-VNNI host (matmulInnerLoopVNNIAsm,
 * simd_amd64.go:41-45; the default here), 1 = amd64 on an AVX2-only host
 * (matmulInnerLoopAsm), 2 = the portable build (noasm tag or another GOARCH:
 * simd_generic.go, matmul_inner_loop_fallback.go, dotProductInline for the
 * attention scores, attention.go:294-298). The three differ only in float32
 * summation order. */
static int g_matmul_path = 0;
void orc_set_matmul_path(int path) { g_matmul_path = path; }

/* Vector inner loops for timing the CPU baseline (orc_set_simd). Off by
 * default: the checker runs the plain loops below. When on, the Q8_0 inner
 * loop of build 0 and the float32 dot product of builds 0 and 1 run as
 * AVX512-VNNI / AVX2 intrinsics that are the reference's assembly instruction
 * for instruction (VPDPBUSD with the zero-point correction, VCVTDQ2PS,
 * VFMADD231PS, the same horizontal sum), so their results are the plain
 * loops' bit for bit; only the speed differs. The switch is ignored on a CPU
 * without AVX512-VNNI. */
static int g_simd = 0;
int orc_set_simd(int on) {
#if defined(__x86_64__) && defined(__GNUC__)
    __builtin_cpu_init();
    g_simd = on && __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl") &&
             __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    (void)on;
    g_simd = 0;
#endif
    return g_simd;
}
static inline uint32_t f32_to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* ------------------------------------------------------------------------
 * f16 → f32 conversions. The reference has two of them and they disagree on
 * subnormals, so both are restated.
 * ---------------------------------------------------------------------- */

/* internal/runtime/model_int8.go:571-597 (used for every projection's block
 * scales via extractQ8_0Scales). The exponent is a uint16 that wraps while
 * normalising a subnormal; the final shift into a uint32 drops the wrapped
 * high bits, which yields the correctly scaled value. */
float orc_f16_runtime(uint16_t f16) {
    uint16_t sign = (f16 >> 15) & 0x1;
    uint16_t exponent = (f16 >> 10) & 0x1f;
    uint16_t fraction = f16 & 0x3ff;
    if (exponent == 0) {
        if (fraction == 0) return bits_to_f32((uint32_t)sign << 31);
        while ((fraction & 0x400) == 0) {
            fraction = (uint16_t)(fraction << 1);
            exponent = (uint16_t)(exponent - 1);
        }
        exponent = (uint16_t)(exponent + 1);
        fraction &= 0x3ff;
    } else if (exponent == 0x1f) {
        return bits_to_f32(((uint32_t)sign << 31) | 0x7f800000u | ((uint32_t)fraction << 13));
    }
    uint32_t exponent32 = (uint32_t)exponent + (127 - 15);
    uint32_t fraction32 = (uint32_t)fraction << 13;
    return bits_to_f32(((uint32_t)sign << 31) | (exponent32 << 23) | fraction32);
}

/* internal/gguf/tensor.go:207-240 (used by ParseQ8_0Block, hence by the token
 * embedding lookup DequantizeQ8_0Row). Subnormals come out at half their true
 * value because the normalising loop starts the exponent at 127-15 without the
 * +1 correction; restated as written. */
float orc_f16_gguf(uint16_t f16) {
    uint32_t sign = (f16 >> 15) & 0x1;
    uint32_t exp = (f16 >> 10) & 0x1f;
    uint32_t mant = f16 & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign << 31;
        } else {
            uint32_t e = 127 - 15;
            uint32_t m = mant;
            while ((m & 0x400) == 0) { m <<= 1; e--; }
            m &= 0x3ff;
            bits = (sign << 31) | (e << 23) | (m << 13);
        }
    } else if (exp == 0x1f) {
        bits = (sign << 31) | (0xffu << 23) | (mant << 13);
    } else {
        bits = (sign << 31) | (((exp - 15 + 127) & 0xff) << 23) | (mant << 13);
    }
    return bits_to_f32(bits);
}

/* ------------------------------------------------------------------------
 * activation.go
 * ---------------------------------------------------------------------- */

/* internal/kernels/activation.go:100-145 */
float orc_fast_exp(float x) {
    const float log2e = 1.442695041f;
    if (x < -10.0f) return 0.0f;
    if (x > 10.0f) return 22026.4657948f;
    float y = x * log2e;
    int32_t intPart = (int32_t)y; /* Go int32(y): truncation toward zero */
    float fracPart = y - (float)intPart;
    const float c1 = 0.693147180559945f;
    const float c2 = 0.240226506959101f;
    const float c3 = 0.055504108664821f;
    const float c4 = 0.009676036358193f;
    float poly = 1.0f + fracPart * (c1 + fracPart * (c2 + fracPart * (c3 + fracPart * c4)));
    if (intPart >= -126 && intPart <= 127) {
        float s = bits_to_f32((uint32_t)(intPart + 127) << 23);
        return poly * s;
    } else if (intPart < -126) {
        return 0.0f;
    }
    return 3.402823e+38f;
}

/* internal/kernels/activation.go:161-213 */
void orc_softmax(float *dst, const float *src, int n) {
    if (n == 0) return;
    float maxVal = src[0];
    for (int i = 1; i < n; i++)
        if (src[i] > maxVal) maxVal = src[i];
    float sum = 0.0f;
    int i = 0;
    for (; i + 3 < n; i += 4) {
        float e0 = orc_fast_exp(src[i] - maxVal);
        float e1 = orc_fast_exp(src[i + 1] - maxVal);
        float e2 = orc_fast_exp(src[i + 2] - maxVal);
        float e3 = orc_fast_exp(src[i + 3] - maxVal);
        dst[i] = e0; dst[i + 1] = e1; dst[i + 2] = e2; dst[i + 3] = e3;
        sum += ((e0 + e1) + e2) + e3;
    }
    for (; i < n; i++) {
        float e = orc_fast_exp(src[i] - maxVal);
        dst[i] = e;
        sum += e;
    }
    if (sum == 0.0f) {
        float inv = 1.0f / (float)n;
        for (int k = 0; k < n; k++) dst[k] = inv;
        return;
    }
    float invSum = 1.0f / sum;
    for (int k = 0; k < n; k++) dst[k] *= invSum;
}

/* internal/kernels/activation.go:47-95 (both the 8-wide body and the tail run
 * the same scalar formula) */
void orc_gelu_quick_simd(float *dst, const float *src, int n) {
    const float scale = 1.702f;
    for (int i = 0; i < n; i++) {
        float x = src[i];
        float sx = scale * x;
        float sig;
        if (sx >= 0.0f) {
            float e = orc_fast_exp(-sx);
            sig = 1.0f / (1.0f + e);
        } else {
            float e = orc_fast_exp(sx);
            sig = e / (1.0f + e);
        }
        dst[i] = x * sig;
    }
}

/* ------------------------------------------------------------------------
 * dot products and norms
 * ---------------------------------------------------------------------- */

/* Horizontal sum used by every AVX2 kernel in the reference:
 * VEXTRACTF128 + VADDPS, then VHADDPS twice (simd_amd64.s:45-51). */
static inline float hsum8(const float acc[8]) {
    float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5], s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
    return (s0 + s1) + (s2 + s3);
}

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
/* VEXTRACTF128 + VADDPS + VHADDPS + VHADDPS (simd_amd64.s:45-51). */
__attribute__((target("avx2,fma"))) static inline float hsum256(__m256 acc) {
    __m128 s4 = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    s4 = _mm_hadd_ps(s4, s4);
    s4 = _mm_hadd_ps(s4, s4);
    return _mm_cvtss_f32(s4);
}

/* dotProductAVX2Asm (simd_amd64.s:19-76): 8 fused lane accumulators, the
 * horizontal sum, then the unfused scalar tail. */
__attribute__((target("avx2,fma"))) static float dot_f32_avx2(const float *a, const float *b, int n) {
    __m256 acc = _mm256_setzero_ps();
    int nv = n / 8;
    for (int v = 0; v < nv; v++) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + 8 * v), _mm256_loadu_ps(b + 8 * v), acc);
    float s = hsum256(acc);
    for (int i = nv * 8; i < n; i++) {
        float p = a[i] * b[i];
        s = s + p;
    }
    return s;
}

/* matmulInnerLoopVNNIAsm (simd_amd64.s:241-304), instruction for instruction. */
__attribute__((target("avx512vnni,avx512vl,avx512bw,avx512f,avx2,fma"))) static float q8_inner_vnni(
    const int8_t *in, const uint8_t *w, const float *scales, int nblocks) {
    const __m256i sign = _mm256_set1_epi8((char)0x80), ones = _mm256_set1_epi8(1);
    __m256 acc = _mm256_setzero_ps();
    for (int b = 0; b < nblocks; b++) {
        const __m256 sc = _mm256_set1_ps(scales[b]);
        const __m256i x = _mm256_loadu_si256((const __m256i *)(in + 32 * b));
        const __m256i q = _mm256_loadu_si256((const __m256i *)(w + 34 * b + 2));
        __m256i d = _mm256_dpbusd_epi32(_mm256_setzero_si256(), _mm256_xor_si256(q, sign), x); /* (w + 128) * x */
        const __m256i sx = _mm256_dpbusd_epi32(_mm256_setzero_si256(), ones, x);             /* sum(x) */
        d = _mm256_sub_epi32(d, _mm256_slli_epi32(sx, 7));
        acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(d), sc, acc);
    }
    return hsum256(acc);
}
#define ORC_HAVE_SIMD 1
#endif

/* dotProductSIMD (simd_amd64.go:59-76): AVX2 assembly when n >= 8
 * (simd_amd64.s:19-76: 8 fused lane accumulators over n/8 vectors, horizontal
 * sum, then an unfused scalar tail), scalar loop otherwise. */
float orc_dot_f32(const float *a, const float *b, int n) {
    if (n == 0) return 0.0f;
#ifdef ORC_HAVE_SIMD
    if (g_simd && n >= 8 && g_matmul_path != 2) return dot_f32_avx2(a, b, n);
#endif
    if (n < 8 || g_matmul_path == 2) { /* dotProductScalar / sumSquaresScalar (simd_generic.go, norm.go:94-100) */
        float s = 0.0f;
        for (int i = 0; i < n; i++) s += a[i] * b[i];
        return s;
    }
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int nv = n / 8;
    for (int v = 0; v < nv; v++)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[8 * v + l], b[8 * v + l], acc[l]);
    float s = hsum8(acc);
    for (int i = nv * 8; i < n; i++) {
        float p = a[i] * b[i];
        s = s + p;
    }
    return s;
}

/* dotProductInline (internal/kernels/attention.go:316-341): the attention score
 * dot product of builds without AVX2. */
static float dot_inline(const float *a, const float *b, int n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        s0 += ((a[i] * b[i] + a[i + 1] * b[i + 1]) + a[i + 2] * b[i + 2]) + a[i + 3] * b[i + 3];
        s1 += ((a[i + 4] * b[i + 4] + a[i + 5] * b[i + 5]) + a[i + 6] * b[i + 6]) + a[i + 7] * b[i + 7];
        s2 += ((a[i + 8] * b[i + 8] + a[i + 9] * b[i + 9]) + a[i + 10] * b[i + 10]) + a[i + 11] * b[i + 11];
        s3 += ((a[i + 12] * b[i + 12] + a[i + 13] * b[i + 13]) + a[i + 14] * b[i + 14]) + a[i + 15] * b[i + 15];
    }
    for (; i + 4 <= n; i += 4) s0 += ((a[i] * b[i] + a[i + 1] * b[i + 1]) + a[i + 2] * b[i + 2]) + a[i + 3] * b[i + 3];
    for (; i < n; i++) s0 += a[i] * b[i];
    return (s0 + s1) + (s2 + s3);
}

/* internal/kernels/norm.go:8-36 (AVX2 branch: VecScaleF32 then VecMulF32, two
 * rounded multiplies per element). */
void orc_rmsnorm(float *dst, const float *src, const float *w, int n, float eps) {
    float sumSq;
    if (n >= 8) {
        sumSq = orc_dot_f32(src, src, n);
    } else {
        sumSq = 0.0f;
        for (int i = 0; i < n; i++) sumSq += src[i] * src[i];
    }
    float meanSq = sumSq / (float)n;
    float rms = (float)sqrt((double)(meanSq + eps));
    float invRms = 1.0f / rms;
    for (int i = 0; i < n; i++) {
        float t = src[i] * invRms;
        dst[i] = t * w[i];
    }
}

/* ------------------------------------------------------------------------
 * INT8 quantisation and the Q8_0 × INT8 matmul
 * ---------------------------------------------------------------------- */

/* QuantizeSymmetricINT8Into + absMaxScalar + quantizeInto
 * (internal/kernels/quantize.go:29-69, :80-90, :92-103). One scale for the
 * whole buffer; round half away from zero of the exact double product. */
void orc_quantize_sym_int8(const float *x, int64_t n, int8_t *codes, float *scale) {
    if (n == 0) { *scale = 1.0f; return; }
    float maxVal = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        float a = bits_to_f32(f32_to_bits(x[i]) & 0x7fffffffu);
        if (a > maxVal) maxVal = a;
    }
    if (maxVal == 0.0f) {
        memset(codes, 0, (size_t)n);
        *scale = 1.0f;
        return;
    }
    float s = maxVal / 127.0f;
    float inv = 1.0f / s;
    for (int64_t i = 0; i < n; i++) {
        double scaled = (double)x[i] * (double)inv;
        double r = round(scaled); /* math.Round: half away from zero */
        int32_t q;
        if (r > 127.0) q = 127;
        else if (r < -127.0) q = -127;
        else q = (int32_t)r;
        codes[i] = (int8_t)q;
    }
    *scale = s;
}

/* extractQ8_0Scales (internal/runtime/model_int8.go:543-569) */
void orc_extract_q8_0_scales(const uint8_t *data, int64_t rows, int cols, float *scales) {
    int bpr = (cols + 31) / 32;
    for (int64_t r = 0; r < rows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *p = data + (size_t)r * bpr * 34 + (size_t)b * 34;
            scales[r * bpr + b] = orc_f16_runtime((uint16_t)(p[0] | (p[1] << 8)));
        }
}

/* Both inner loops (internal/kernels/simd_amd64.s:164-237 and :241-304) keep 8
 * float accumulators; per 32-byte block, lane l receives an exact int32 sum of
 * 4 products, converted to float and FMA'd with the block scale, and the lanes
 * are summed horizontally at the end. They differ only in which 4 products a
 * lane holds: VNNI (VPDPBUSD) sums the consecutive bytes 4l..4l+3; AVX2
 * (VPMOVSXBW + VPMADDWD on each 16-byte half, then VPADDD) sums bytes 2l, 2l+1,
 * 16+2l, 17+2l. */
static float q8_inner_loop(const int8_t *in, const uint8_t *w, const float *scales, int nblocks) {
    if (g_matmul_path == 2) { /* matmul_inner_loop_fallback.go:16-39 */
        float sum = 0.0f;
        for (int b = 0; b < nblocks; b++) {
            const int8_t *x = in + 32 * b;
            const int8_t *q = (const int8_t *)(w + 34 * b + 2);
            int32_t acc = 0;
            for (int t = 0; t < 32; t++) acc += (int32_t)x[t] * (int32_t)q[t];
            float p = (float)acc * scales[b];
            sum = sum + p;
        }
        return sum;
    }
#ifdef ORC_HAVE_SIMD
    if (g_simd && g_matmul_path == 0) return q8_inner_vnni(in, w, scales, nblocks);
#endif
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < nblocks; b++) {
        const int8_t *x = in + 32 * b;
        const int8_t *q = (const int8_t *)(w + 34 * b + 2);
        float sc = scales[b];
        for (int l = 0; l < 8; l++) {
            int32_t s = 0;
            if (g_matmul_path == 1) {
                s = (int32_t)x[2 * l] * q[2 * l] + (int32_t)x[2 * l + 1] * q[2 * l + 1] +
                    (int32_t)x[16 + 2 * l] * q[16 + 2 * l] + (int32_t)x[17 + 2 * l] * q[17 + 2 * l];
            } else {
                for (int t = 0; t < 4; t++) s += (int32_t)x[4 * l + t] * (int32_t)q[4 * l + t];
            }
            acc[l] = fmaf((float)s, sc, acc[l]);
        }
    }
    return hsum8(acc);
}

/* MatMulQ8_0INT8 → matMulQ8_0INT8SerialRange (quantize.go:346-369, :390-458):
 * dst[i,j] = inputScale * (inner loop over full blocks + partial-block tail). */
void orc_matmul_q8_0_int8(float *dst, const uint8_t *w_q8, const float *w_scales, const int8_t *a,
                          float a_scale, int batch, int in_dim, int out_dim) {
    int bpr = (in_dim + 31) / 32;
    int bytes_per_row = bpr * 34;
    int full = in_dim / 32;
    int tail = in_dim - full * 32;
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && (int64_t)batch * out_dim > 4096)
    for (int j = 0; j < out_dim; j++) {
        const uint8_t *wrow = w_q8 + (size_t)j * bytes_per_row;
        const float *srow = w_scales + (size_t)j * bpr;
        for (int i = 0; i < batch; i++) {
            const int8_t *arow = a + (size_t)i * in_dim;
            float sum = 0.0f;
            if (full > 0) sum = q8_inner_loop(arow, wrow, srow, full);
            if (tail) {
                const int8_t *q = (const int8_t *)(wrow + full * 34 + 2);
                int32_t bs = 0;
                for (int t = 0; t < tail; t++) bs += (int32_t)arow[full * 32 + t] * (int32_t)q[t];
                float p = (float)bs * srow[full];
                sum = sum + p;
            }
            dst[(size_t)i * out_dim + j] = sum * a_scale;
        }
    }
}

/* ------------------------------------------------------------------------
 * GGUF v3 reader (internal/gguf/reader.go:98-178, format.go)
 * ---------------------------------------------------------------------- */

typedef struct {
    char name[96];
    uint32_t dtype;
    uint32_t ndim;
    uint64_t dims[4];
    uint64_t offset;
    uint64_t size;
} orc_tensor;

typedef struct {
    const uint8_t *data;
    size_t len;
    size_t data_off;
    int ntensors;
    orc_tensor *tensors;
    /* metadata we consume (model.go:424-517) */
    char arch[64];
    int has_embed, has_blocks, has_heads, has_heads_kv, has_ff, has_ctx, has_eps, has_rope;
    uint32_t embed, blocks, heads, heads_kv, ff, ctx;
    float eps, rope;
    int64_t ntokens; /* length of tokenizer.ggml.tokens, -1 if absent */
} orc_gguf;

static uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }
static uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }

static int dtype_block_size(uint32_t d) { /* format.go:86-117 */
    switch (d) {
    case 0: return 4; case 1: return 2; case 2: return 18; case 3: return 20; case 6: return 22;
    case 7: return 24; case 8: return 34; case 9: return 36; case 16: return 1; case 17: return 2;
    case 18: return 4; case 19: return 8; case 20: return 8; default: return 0;
    }
}
static int dtype_elems_per_block(uint32_t d) { /* format.go:120-131 */
    switch (d) {
    case 0: case 1: case 16: case 17: case 18: case 19: case 20: return 1;
    case 2: case 3: case 6: case 7: return 16;
    case 8: case 9: return 32;
    default: return 0;
    }
}

/* Skips one metadata value of type t at *off (reader.go:220-271); when the
 * value is a uint32/float32/string it is also returned through the outputs. */
static int gguf_value(const uint8_t *d, size_t len, size_t *off, uint32_t t, uint32_t *u32, float *f32,
                      const char **s, uint64_t *slen, int64_t *arrlen) {
    size_t o = *off;
#define NEED(k) do { if (o + (k) > len) return -1; } while (0)
    switch (t) {
    case 0: case 1: case 7: NEED(1); o += 1; break;
    case 2: case 3: NEED(2); o += 2; break;
    case 4: NEED(4); if (u32) *u32 = rd32(d + o); o += 4; break;
    case 5: NEED(4); o += 4; break;
    case 6: NEED(4); if (f32) *f32 = bits_to_f32(rd32(d + o)); o += 4; break;
    case 10: case 11: case 12: NEED(8); o += 8; break;
    case 8: {
        NEED(8);
        uint64_t n = rd64(d + o); o += 8; NEED(n);
        if (s) { *s = (const char *)(d + o); *slen = n; }
        o += n;
        break;
    }
    case 9: {
        NEED(12);
        uint32_t at = rd32(d + o); o += 4;
        uint64_t n = rd64(d + o); o += 8;
        if (arrlen) *arrlen = (int64_t)n;
        for (uint64_t i = 0; i < n; i++)
            if (gguf_value(d, len, &o, at, NULL, NULL, NULL, NULL, NULL)) return -1;
        break;
    }
    default: return -1;
    }
#undef NEED
    *off = o;
    return 0;
}

static int gguf_parse(orc_gguf *g, char *err, int errlen) {
    const uint8_t *d = g->data;
    size_t len = g->len, o = 0;
    if (len < 24) { seterr(err, errlen, "file too small for header"); return -1; }
    uint32_t magic = rd32(d);
    if (magic != 0x46554747u) { seterr(err, errlen, "invalid magic: 0x%08x", magic); return -1; }
    uint32_t ver = rd32(d + 4);
    if (ver != 3) { seterr(err, errlen, "unsupported version: %u", ver); return -1; }
    uint64_t nt = rd64(d + 8), nkv = rd64(d + 16);
    o = 24;
    g->ntokens = -1;
    for (uint64_t i = 0; i < nkv; i++) {
        if (o + 8 > len) goto trunc;
        uint64_t kl = rd64(d + o); o += 8;
        if (o + kl + 4 > len) goto trunc;
        char key[256];
        size_t kc = kl < 255 ? kl : 255;
        memcpy(key, d + o, kc); key[kc] = 0;
        o += kl;
        uint32_t t = rd32(d + o); o += 4;
        uint32_t u = 0; float f = 0; const char *s = NULL; uint64_t sl = 0; int64_t al = -1;
        if (gguf_value(d, len, &o, t, &u, &f, &s, &sl, &al)) goto trunc;
        if (!strcmp(key, "general.architecture") && t == 8) {
            size_t c = sl < 63 ? sl : 63; memcpy(g->arch, s, c); g->arch[c] = 0;
        } else if (!strcmp(key, "tokenizer.ggml.tokens") && t == 9) {
            g->ntokens = al;
        } else {
            const char *dot = strchr(key, '.');
            const char *sub = dot ? dot + 1 : key;
            /* keys are "<arch>.<name>"; the arch is matched after parsing */
            if (t == 4) {
                if (!strcmp(sub, "embedding_length")) { g->embed = u; g->has_embed = 1; }
                else if (!strcmp(sub, "block_count")) { g->blocks = u; g->has_blocks = 1; }
                else if (!strcmp(sub, "attention.head_count")) { g->heads = u; g->has_heads = 1; }
                else if (!strcmp(sub, "attention.head_count_kv")) { g->heads_kv = u; g->has_heads_kv = 1; }
                else if (!strcmp(sub, "feed_forward_length")) { g->ff = u; g->has_ff = 1; }
                else if (!strcmp(sub, "context_length")) { g->ctx = u; g->has_ctx = 1; }
            } else if (t == 6) {
                if (!strcmp(sub, "attention.layer_norm_rms_epsilon")) { g->eps = f; g->has_eps = 1; }
                else if (!strcmp(sub, "rope.freq_base")) { g->rope = f; g->has_rope = 1; }
            }
        }
    }
    g->ntensors = (int)nt;
    g->tensors = (orc_tensor *)calloc(nt ? nt : 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < nt; i++) {
        orc_tensor *tt = &g->tensors[i];
        if (o + 8 > len) goto trunc;
        uint64_t nl = rd64(d + o); o += 8;
        if (o + nl + 4 > len) goto trunc;
        size_t c = nl < 95 ? nl : 95;
        memcpy(tt->name, d + o, c); tt->name[c] = 0;
        o += nl;
        tt->ndim = rd32(d + o); o += 4;
        if (tt->ndim > 4 || o + 8 * tt->ndim + 12 > len) goto trunc;
        uint64_t total = 1;
        for (uint32_t k = 0; k < tt->ndim; k++) { tt->dims[k] = rd64(d + o); o += 8; total *= tt->dims[k]; }
        tt->dtype = rd32(d + o); o += 4;
        tt->offset = rd64(d + o); o += 8;
        int bs = dtype_block_size(tt->dtype), epb = dtype_elems_per_block(tt->dtype);
        if (epb > 0 && bs > 0) tt->size = (total + epb - 1) / epb * bs;
        else tt->size = total * bs;
    }
    g->data_off = (o + 31) & ~(size_t)31; /* reader.go:175: fixed 32-byte alignment */
    return 0;
trunc:
    seterr(err, errlen, "truncated GGUF file");
    return -1;
}

static const orc_tensor *gguf_find(const orc_gguf *g, const char *name) {
    for (int i = 0; i < g->ntensors; i++)
        if (!strcmp(g->tensors[i].name, name)) return &g->tensors[i];
    return NULL;
}

static const uint8_t *gguf_data(const orc_gguf *g, const orc_tensor *t) {
    size_t off = g->data_off + t->offset;
    if (off + t->size > g->len) return NULL;
    return g->data + off;
}

/* ------------------------------------------------------------------------
 * Model (internal/runtime)
 * ---------------------------------------------------------------------- */

typedef struct {
    const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;      /* raw Q8_0 views */
    float *sq, *sk, *sv, *so, *sg, *su, *sd;               /* extracted scales */
    const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm;
} orc_layer;

struct orc_model {
    orc_gguf g;
    void *map;
    size_t maplen;
    orc_config cfg;
    const uint8_t *tok_embd;
    const float *output_norm;
    orc_layer *layers;
    float *rope_cos, *rope_sin; /* [max_seq_len][head_dim/2] */
    /* model-faithful extensions (orc_model_set_faithful; the reference has
     * neither): sliding-window layers with their own RoPE tables, and the
     * dense 2/3 head after pooling */
    int swa_window, swa_pattern, dense_head;
    float *rope_cos_swa, *rope_sin_swa;
    const uint8_t *dense2, *dense3;
    float *sd2, *sd3;
    int dense_mid; /* dense_2 output width */
};

void orc_model_config(const orc_model *m, orc_config *out) { *out = m->cfg; }

static void rope_tables(const orc_config *c, float base, float **cs, float **sn);

/* Model-faithful mode (no reference counterpart; the reference runs full
 * attention in every layer and has no dense head, model_int8.go:235-255,
 * :500): sliding-window layers, their RoPE base, the dense 2/3 head. All
 * zero: the reference's forward. Returns -1 if the head is asked for and the
 * file has no dense_2/dense_3 weights. */
int orc_model_set_faithful(orc_model *m, int swa_window, int swa_pattern, float rope_base_swa, int dense_head) {
    if (dense_head && !(m->dense2 && m->dense3 && m->sd2 && m->sd3)) return -1;
    m->swa_window = swa_window > 0 ? swa_window : 0;
    m->swa_pattern = swa_pattern > 0 ? swa_pattern : 0;
    m->dense_head = dense_head ? 1 : 0;
    free(m->rope_cos_swa); free(m->rope_sin_swa);
    m->rope_cos_swa = m->rope_sin_swa = NULL;
    if (m->swa_window && rope_base_swa > 0.0f && rope_base_swa != m->cfg.rope_base)
        rope_tables(&m->cfg, rope_base_swa, &m->rope_cos_swa, &m->rope_sin_swa);
    return 0;
}

static const float *load_f32(const orc_gguf *g, const char *name) {
    const orc_tensor *t = gguf_find(g, name);
    if (!t || t->dtype != 0) return NULL; /* synthetic models store norms as F32 */
    return (const float *)gguf_data(g, t);
}

static const uint8_t *load_q8(const orc_gguf *g, const char *name, char *err, int errlen) {
    const orc_tensor *t = gguf_find(g, name);
    if (!t) { seterr(err, errlen, "tensor not found: %s", name); return NULL; }
    if (t->dtype != 8) { seterr(err, errlen, "expected Q8_0 for %s", name); return NULL; }
    const uint8_t *p = gguf_data(g, t);
    if (!p) seterr(err, errlen, "tensor data out of bounds: %s", name);
    return p;
}

/* NewRoPECache (rope_cache.go:15-44): cos/sin of float32(p) * float32 freq. */
static void rope_tables(const orc_config *c, float base, float **cs, float **sn) {
    int half = c->head_dim / 2;
    *cs = (float *)malloc(sizeof(float) * (size_t)c->max_seq_len * half);
    *sn = (float *)malloc(sizeof(float) * (size_t)c->max_seq_len * half);
    float *freqs = (float *)malloc(sizeof(float) * half);
    for (int i = 0; i < half; i++)
        freqs[i] = (float)(1.0 / pow((double)base, (double)(2 * i) / (double)c->head_dim));
    for (int p = 0; p < c->max_seq_len; p++) {
        float pf = (float)p;
        for (int i = 0; i < half; i++) {
            float theta = pf * freqs[i];
            (*cs)[(size_t)p * half + i] = (float)cos((double)theta);
            (*sn)[(size_t)p * half + i] = (float)sin((double)theta);
        }
    }
    free(freqs);
}

static float *scales_for(const uint8_t *w, int64_t bytes, int cols) {
    int bpr = (cols + 31) / 32;
    int64_t rows = bytes / (bpr * 34);
    float *s = (float *)malloc(sizeof(float) * (size_t)(rows * bpr));
    orc_extract_q8_0_scales(w, rows, cols, s);
    return s;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    if (m->layers) {
        for (int l = 0; l < m->cfg.num_layers; l++) {
            orc_layer *L = &m->layers[l];
            free(L->sq); free(L->sk); free(L->sv); free(L->so); free(L->sg); free(L->su); free(L->sd);
        }
        free(m->layers);
    }
    free(m->rope_cos); free(m->rope_sin);
    free(m->rope_cos_swa); free(m->rope_sin_swa);
    free(m->sd2); free(m->sd3);
    free(m->g.tensors);
    if (m->map) munmap(m->map, m->maplen);
    free(m);
}

orc_model *orc_model_load(const char *path, char *err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { seterr(err, errlen, "open file: %s", path); return NULL; }
    struct stat st;
    fstat(fd, &st);
    void *map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { seterr(err, errlen, "mmap file"); return NULL; }
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->map = map; m->maplen = (size_t)st.st_size;
    m->g.data = (const uint8_t *)map; m->g.len = (size_t)st.st_size;
    if (gguf_parse(&m->g, err, errlen)) { orc_model_free(m); return NULL; }
    orc_gguf *g = &m->g;
    /* parseConfig (model.go:424-517) */
    orc_config *c = &m->cfg;
    c->norm_eps = 1e-6f; c->rope_base = 10000.0f; c->max_seq_len = 2048;
    if (!g->has_embed) { seterr(err, errlen, "%s.embedding_length not found", g->arch); orc_model_free(m); return NULL; }
    if (!g->has_blocks) { seterr(err, errlen, "%s.block_count not found", g->arch); orc_model_free(m); return NULL; }
    if (!g->has_heads) { seterr(err, errlen, "%s.attention.head_count not found", g->arch); orc_model_free(m); return NULL; }
    c->embed_dim = (int)g->embed; c->num_layers = (int)g->blocks; c->num_heads = (int)g->heads;
    c->num_kv_heads = g->has_heads_kv ? (int)g->heads_kv : c->num_heads;
    c->head_dim = c->embed_dim / c->num_heads;
    c->attention_scale = 1.0f / (float)sqrt((double)c->head_dim);
    if (g->has_ff) c->interm_dim = (int)g->ff;
    else c->interm_dim = c->embed_dim * 3;
    if (g->has_ctx) c->max_seq_len = (int)g->ctx;
    if (g->has_eps) c->norm_eps = g->eps;
    if (g->has_rope) c->rope_base = g->rope;
    c->vocab_size = g->ntokens >= 0 ? (int)g->ntokens : g->ntensors;
    /* loadWeights (model.go:520-552) */
    m->tok_embd = load_q8(g, "token_embd.weight", err, errlen);
    if (!m->tok_embd) { orc_model_free(m); return NULL; }
    m->output_norm = load_f32(g, "output_norm.weight");
    /* NewRoPECache (rope_cache.go:15-44) */
    rope_tables(c, c->rope_base, &m->rope_cos, &m->rope_sin);
    /* the dense head's weights, when the file has them (not read by the
     * reference; used only in the model-faithful mode) */
    {
        const orc_tensor *t2 = gguf_find(g, "dense_2.weight"), *t3 = gguf_find(g, "dense_3.weight");
        if (t2 && t3 && t2->dtype == 8 && t3->dtype == 8 && t2->ndim == 2 && t3->ndim == 2 &&
            t2->dims[0] == (uint64_t)c->embed_dim && t3->dims[1] == (uint64_t)c->embed_dim &&
            t3->dims[0] == t2->dims[1]) {
            m->dense2 = gguf_data(g, t2);
            m->dense3 = gguf_data(g, t3);
            m->dense_mid = (int)t2->dims[1];
            if (m->dense2 && m->dense3) {
                m->sd2 = scales_for(m->dense2, (int64_t)t2->size, c->embed_dim);
                m->sd3 = scales_for(m->dense3, (int64_t)t3->size, m->dense_mid);
            }
        }
    }
    /* loadLayerINT8 (model_int8.go:54-119) */
    m->layers = (orc_layer *)calloc((size_t)c->num_layers, sizeof(orc_layer));
    for (int l = 0; l < c->num_layers; l++) {
        orc_layer *L = &m->layers[l];
        char nm[96];
#define F32(field, suffix) snprintf(nm, sizeof nm, "blk.%d.%s", l, suffix); L->field = load_f32(g, nm);
        F32(attn_norm, "attn_norm.weight");
        F32(ffn_norm, "ffn_norm.weight");
        if (!L->attn_norm || !L->ffn_norm) { seterr(err, errlen, "tensor not found: blk.%d norm", l); orc_model_free(m); return NULL; }
        F32(q_norm, "attn_q_norm.weight");
        F32(k_norm, "attn_k_norm.weight");
        F32(post_attn_norm, "post_attention_norm.weight");
        F32(post_ffw_norm, "post_ffw_norm.weight");
#undef F32
#define Q8(field, sfield, suffix, cols)                                              \
        snprintf(nm, sizeof nm, "blk.%d.%s", l, suffix);                             \
        L->field = load_q8(g, nm, err, errlen);                                      \
        if (!L->field) { orc_model_free(m); return NULL; }                           \
        L->sfield = scales_for(L->field, (int64_t)gguf_find(g, nm)->size, cols);
        Q8(wq, sq, "attn_q.weight", c->embed_dim);
        Q8(wk, sk, "attn_k.weight", c->embed_dim);
        Q8(wv, sv, "attn_v.weight", c->embed_dim);
        Q8(wo, so, "attn_output.weight", c->embed_dim);
        Q8(wg, sg, "ffn_gate.weight", c->embed_dim);
        Q8(wu, su, "ffn_up.weight", c->embed_dim);
        Q8(wd, sd, "ffn_down.weight", c->interm_dim);
#undef Q8
    }
    return m;
}

/* applyRMSNormParallel (model_int8.go:616-706): an RMSNorm per token row. */
static void norm_rows(float *h, const float *w, int rows, int dim, float eps) {
    for (int i = 0; i < rows; i++) orc_rmsnorm(h + (size_t)i * dim, h + (size_t)i * dim, w, dim, eps);
}

/* RoPE with cached tables (rope_cache.go:117-260, cached branch): NeoX pairs
 * (i, i+half) per head; layout [S][nHeads*headDim]. */
static void rope_apply(const orc_model *m, const float *tcos, const float *tsin, float *qk, int S, int nHeads) {
    int hd = m->cfg.head_dim, half = hd / 2;
    for (int s = 0; s < S; s++) {
        const float *cs = tcos + (size_t)s * half, *sn = tsin + (size_t)s * half;
        for (int h = 0; h < nHeads; h++) {
            float *x = qk + ((size_t)s * nHeads + h) * hd;
            for (int i = 0; i < half; i++) {
                float v0 = x[i], v1 = x[i + half];
                float a = v0 * cs[i], b = v1 * sn[i];
                float c2 = v0 * sn[i], d2 = v1 * cs[i];
                x[i] = a - b;
                x[i + half] = c2 + d2;
            }
        }
    }
}

/* forwardINT8WithDim (internal/runtime/model_int8.go:148-256) with
 * runAttentionINT8 (:349-507) and runMLPINT8 (:510-538). */
int orc_forward(const orc_model *m, const int32_t *ids, int S, int target_dim, float *out, char *err,
                int errlen) {
    const orc_config *c = &m->cfg;
    int H = c->embed_dim, F = c->interm_dim, nh = c->num_heads, nkv = c->num_kv_heads, hd = c->head_dim;
    int kvd = nkv * hd;
    if (target_dim <= 0 || target_dim > H) {
        seterr(err, errlen, "target dimension %d out of range (1..%d)", target_dim, H);
        return -1;
    }
    if (S == 0) { seterr(err, errlen, "empty input"); return -1; }
    if (S > c->max_seq_len) { seterr(err, errlen, "sequence too long: %d > %d", S, c->max_seq_len); return -1; }
    size_t SH = (size_t)S * H;
    float *hidden = (float *)malloc(sizeof(float) * SH);
    float *residual = (float *)malloc(sizeof(float) * SH);
    float *q = (float *)malloc(sizeof(float) * SH);
    float *k = (float *)malloc(sizeof(float) * (size_t)S * kvd);
    float *v = (float *)malloc(sizeof(float) * (size_t)S * kvd);
    float *ke = (float *)malloc(sizeof(float) * SH);
    float *ve = (float *)malloc(sizeof(float) * SH);
    float *attn = (float *)malloc(sizeof(float) * SH);
    float *scores = (float *)malloc(sizeof(float) * (size_t)S * S);
    float *gate = (float *)malloc(sizeof(float) * (size_t)S * F);
    float *up = (float *)malloc(sizeof(float) * (size_t)S * F);
    int8_t *codes = (int8_t *)malloc((size_t)S * (F > H ? F : H));
    float *scaled = (float *)malloc(sizeof(float) * hd);
    int rc = 0;
    /* embedding lookup (:167-178) with gguf.DequantizeQ8_0Row (gguf/tensor.go:157-177) */
    int bpr = (H + 31) / 32;
    for (int i = 0; i < S; i++) {
        int t = ids[i];
        if (t < 0 || t >= c->vocab_size) { seterr(err, errlen, "token ID out of range: %d", t); rc = -1; goto done; }
        const uint8_t *row = m->tok_embd + (size_t)t * bpr * 34;
        for (int b = 0; b < bpr; b++) {
            const uint8_t *blk = row + b * 34;
            float sc = orc_f16_gguf((uint16_t)(blk[0] | (blk[1] << 8)));
            int end = (b + 1) * 32 < H ? (b + 1) * 32 : H;
            for (int e = b * 32; e < end; e++) hidden[(size_t)i * H + e] = (float)(int8_t)blk[2 + e - b * 32] * sc;
        }
    }
    {
        float sf = (float)sqrt((double)H); /* :181-184 */
        for (size_t i = 0; i < SH; i++) hidden[i] *= sf;
    }
    for (int l = 0; l < c->num_layers; l++) {
        const orc_layer *L = &m->layers[l];
        float sc;
        memcpy(residual, hidden, sizeof(float) * SH);
        norm_rows(hidden, L->attn_norm, S, H, c->norm_eps);
        orc_quantize_sym_int8(hidden, (int64_t)SH, codes, &sc);
        /* runAttentionINT8 */
        orc_matmul_q8_0_int8(q, L->wq, L->sq, codes, sc, S, H, H);
        orc_matmul_q8_0_int8(k, L->wk, L->sk, codes, sc, S, H, kvd);
        orc_matmul_q8_0_int8(v, L->wv, L->sv, codes, sc, S, H, kvd);
        if (L->q_norm)
            for (int s = 0; s < S; s++)
                for (int h = 0; h < nh; h++) {
                    float *p = q + (size_t)s * H + (size_t)h * hd;
                    orc_rmsnorm(p, p, L->q_norm, hd, c->norm_eps);
                }
        if (L->k_norm)
            for (int s = 0; s < S; s++)
                for (int h = 0; h < nkv; h++) {
                    float *p = k + (size_t)s * kvd + (size_t)h * hd;
                    orc_rmsnorm(p, p, L->k_norm, hd, c->norm_eps);
                }
        /* model-faithful mode: sliding layers (all but every swa_pattern-th)
         * see keys within swa_window / 2 positions and may use their own RoPE
         * base; otherwise every layer attends to every key (model_int8.go:500) */
        const int sliding = m->swa_window > 0 && m->swa_pattern > 0 && (l + 1) % m->swa_pattern != 0;
        const int hw = sliding ? m->swa_window / 2 : S;
        const float *tc = sliding && m->rope_cos_swa ? m->rope_cos_swa : m->rope_cos;
        const float *ts = sliding && m->rope_sin_swa ? m->rope_sin_swa : m->rope_sin;
        rope_apply(m, tc, ts, q, S, nh);
        rope_apply(m, tc, ts, k, S, nkv);
        /* GQA expand (:455-479) */
        int grp = nh / nkv;
        for (int s = 0; s < S; s++)
            for (int kh = 0; kh < nkv; kh++)
                for (int g2 = 0; g2 < grp; g2++) {
                    int qh = kh * grp + g2;
                    memcpy(ke + (size_t)s * H + (size_t)qh * hd, k + (size_t)s * kvd + (size_t)kh * hd, sizeof(float) * hd);
                    memcpy(ve + (size_t)s * H + (size_t)qh * hd, v + (size_t)s * kvd + (size_t)kh * hd, sizeof(float) * hd);
                }
        /* MultiHeadAttentionChunked, mask nil (attention.go:178-310, :344-363).
         * Query i's row covers keys [lo, hi]: all S keys, or the sliding
         * window, whose keys form a contiguous row of their own for the
         * softmax and the weighted sum. */
        for (int h = 0; h < nh; h++) {
            for (int i = 0; i < S; i++) {
                const int lo = i - hw > 0 ? i - hw : 0, hi = i + hw < S - 1 ? i + hw : S - 1;
                const float *qr = q + (size_t)i * H + (size_t)h * hd;
                for (int j = lo; j <= hi; j++) {
                    const float *kr = ke + (size_t)j * H + (size_t)h * hd;
                    float d = g_matmul_path == 2 ? dot_inline(qr, kr, hd) : orc_dot_f32(qr, kr, hd);
                    scores[(size_t)i * S + (j - lo)] = d * c->attention_scale;
                }
                orc_softmax(scores + (size_t)i * S, scores + (size_t)i * S, hi - lo + 1);
            }
            for (int i = 0; i < S; i++) {
                const int lo = i - hw > 0 ? i - hw : 0, hi = i + hw < S - 1 ? i + hw : S - 1;
                float *o = attn + (size_t)i * H + (size_t)h * hd;
                for (int d = 0; d < hd; d++) o[d] = 0.0f;
                for (int j = lo; j <= hi; j++) {
                    float w = scores[(size_t)i * S + (j - lo)];
                    if (w == 0.0f) continue;
                    const float *vr = ve + (size_t)j * H + (size_t)h * hd;
                    for (int d = 0; d < hd; d++) scaled[d] = vr[d] * w;   /* VecScaleF32 */
                    for (int d = 0; d < hd; d++) o[d] = o[d] + scaled[d]; /* VecAddF32 */
                }
            }
        }
        orc_quantize_sym_int8(attn, (int64_t)SH, codes, &sc);
        orc_matmul_q8_0_int8(hidden, L->wo, L->so, codes, sc, S, H, H);
        if (L->post_attn_norm) norm_rows(hidden, L->post_attn_norm, S, H, c->norm_eps);
        for (size_t i = 0; i < SH; i++) hidden[i] += residual[i];
        memcpy(residual, hidden, sizeof(float) * SH);
        norm_rows(hidden, L->ffn_norm, S, H, c->norm_eps);
        orc_quantize_sym_int8(hidden, (int64_t)SH, codes, &sc);
        /* runMLPINT8 */
        orc_matmul_q8_0_int8(gate, L->wg, L->sg, codes, sc, S, H, F);
        orc_matmul_q8_0_int8(up, L->wu, L->su, codes, sc, S, H, F);
        orc_gelu_quick_simd(gate, gate, S * F);
        for (size_t i = 0; i < (size_t)S * F; i++) gate[i] = gate[i] * up[i];
        orc_quantize_sym_int8(gate, (int64_t)S * F, codes, &sc);
        orc_matmul_q8_0_int8(hidden, L->wd, L->sd, codes, sc, S, F, H);
        if (L->post_ffw_norm) norm_rows(hidden, L->post_ffw_norm, S, H, c->norm_eps);
        for (size_t i = 0; i < SH; i++) hidden[i] += residual[i];
    }
    if (m->output_norm) norm_rows(hidden, m->output_norm, S, H, c->norm_eps);
    {
        /* MeanPoolingPartial (attention.go:423-445) + l2Normalize (model.go:808-820) */
        int od = target_dim;
        if (m->dense_head) {
            /* model-faithful head: pool every channel, dense_2 then dense_3
             * (Q8_0, each input quantised as one INT8 buffer like every
             * projection of the forward), then the first od outputs */
            float *pool = (float *)malloc(sizeof(float) * H), *y1 = (float *)malloc(sizeof(float) * m->dense_mid),
                  *y2 = (float *)malloc(sizeof(float) * H);
            int8_t *pc = (int8_t *)malloc((size_t)(m->dense_mid > H ? m->dense_mid : H));
            for (int i = 0; i < H; i++) pool[i] = 0.0f;
            for (int s = 0; s < S; s++)
                for (int i = 0; i < H; i++) pool[i] += hidden[(size_t)s * H + i];
            float invS = 1.0f / (float)S, sc2;
            for (int i = 0; i < H; i++) pool[i] *= invS;
            orc_quantize_sym_int8(pool, H, pc, &sc2);
            orc_matmul_q8_0_int8(y1, m->dense2, m->sd2, pc, sc2, 1, H, m->dense_mid);
            orc_quantize_sym_int8(y1, m->dense_mid, pc, &sc2);
            orc_matmul_q8_0_int8(y2, m->dense3, m->sd3, pc, sc2, 1, m->dense_mid, H);
            for (int i = 0; i < od; i++) out[i] = y2[i];
            free(pool); free(y1); free(y2); free(pc);
        } else {
        for (int i = 0; i < od; i++) out[i] = 0.0f;
        for (int s = 0; s < S; s++)
            for (int i = 0; i < od; i++) out[i] += hidden[(size_t)s * H + i];
        float inv = 1.0f / (float)S;
        for (int i = 0; i < od; i++) out[i] *= inv;
        }
        float ss = 0.0f;
        for (int i = 0; i < od; i++) ss += out[i] * out[i];
        if (ss != 0.0f) {
            float nrm = (float)sqrt((double)ss);
            for (int i = 0; i < od; i++) out[i] /= nrm;
        }
    }
done:
    free(hidden); free(residual); free(q); free(k); free(v); free(ke); free(ve); free(attn);
    free(scores); free(gate); free(up); free(codes); free(scaled);
    return rc;
}

int orc_forward_batch(const orc_model *m, const int32_t *ids, const int32_t *offsets, int nseq,
                      int target_dim, float *out, int nthreads, char *err, int errlen) {
    int rc = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    (void)nthreads;
#endif
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
    for (int s = 0; s < nseq; s++) {
        char e2[256];
        int r = orc_forward(m, ids + offsets[s], offsets[s + 1] - offsets[s], target_dim,
                            out + (size_t)s * target_dim, e2, sizeof e2);
        if (r) {
#pragma omp critical
            {
                if (!rc) { rc = r; seterr(err, errlen, "%s", e2); }
            }
        }
    }
    return rc;
}

/* ------------------------------------------------------------------------
 * search/brute
 * ---------------------------------------------------------------------- */

/* builder.go:129-141: float64 sum of float32 squares, float32 inverse norm. */
void orc_normalize(float *v, int n) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) { float p = v[i] * v[i]; sum += (double)p; }
    if (sum == 0.0) return;
    float norm = (float)(1.0 / sqrt(sum));
    for (int i = 0; i < n; i++) v[i] *= norm;
}

/* quant.go:17-28 */
void orc_quantize_int8_vec(const float *v, int n, int8_t *out) {
    for (int i = 0; i < n; i++) {
        float x = v[i];
        if (x > 1.0f) x = 1.0f; else if (x < -1.0f) x = -1.0f;
        out[i] = (int8_t)(int32_t)round((double)x * 127.0);
    }
}

/* quant.go:30-41 */
void orc_quantize_int16_vec(const float *v, int n, int16_t *out) {
    for (int i = 0; i < n; i++) {
        float x = v[i];
        if (x > 1.0f) x = 1.0f; else if (x < -1.0f) x = -1.0f;
        out[i] = (int16_t)(int32_t)round((double)x * 32767.0);
    }
}

static const float INV127 = 0.0078740157f;     /* dot_amd64.s:5, quant.go:57 */
static const float INV32767 = 0.000030518509f; /* dot_amd64.s:8, quant.go:64 */

/* dotInt8 (quant.go:83-108): dotInt8AVX2 on the dim&^7 prefix
 * (dot_amd64.s:12-43: code*inv127, then *query, unfused adds into 8 lanes),
 * then a 4-way unrolled LUT tail. */
float orc_dot_int8_ref(const int8_t *v, const float *q, int dim) {
    float sum = 0.0f;
    int start = 0;
    if (dim >= 8) {
        int n = dim & ~7;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int b = 0; b < n; b += 8)
            for (int l = 0; l < 8; l++) {
                float t = (float)v[b + l] * INV127;
                t = t * q[b + l];
                acc[l] = acc[l] + t;
            }
        sum += hsum8(acc);
        start = n;
    }
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = start;
    for (; i + 4 <= dim; i += 4) {
        int8_t c0 = v[i] < -127 ? -127 : v[i], c1 = v[i + 1] < -127 ? -127 : v[i + 1];
        int8_t c2 = v[i + 2] < -127 ? -127 : v[i + 2], c3 = v[i + 3] < -127 ? -127 : v[i + 3];
        s0 += q[i] * ((float)c0 * INV127);
        s1 += q[i + 1] * ((float)c1 * INV127);
        s2 += q[i + 2] * ((float)c2 * INV127);
        s3 += q[i + 3] * ((float)c3 * INV127);
    }
    sum += ((s0 + s1) + s2) + s3;
    for (; i < dim; i++) {
        int8_t c = v[i] < -127 ? -127 : v[i];
        sum += q[i] * ((float)c * INV127);
    }
    return sum;
}

/* dotInt16 (quant.go:110-135, dot_amd64.s:46-77) */
float orc_dot_int16_ref(const int16_t *v, const float *q, int dim) {
    float sum = 0.0f;
    int start = 0;
    if (dim >= 8) {
        int n = dim & ~7;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int b = 0; b < n; b += 8)
            for (int l = 0; l < 8; l++) {
                float t = (float)v[b + l] * INV32767;
                t = t * q[b + l];
                acc[l] = acc[l] + t;
            }
        sum += hsum8(acc);
        start = n;
    }
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = start;
    for (; i + 4 <= dim; i += 4) {
        int16_t c0 = v[i] < -32767 ? -32767 : v[i], c1 = v[i + 1] < -32767 ? -32767 : v[i + 1];
        int16_t c2 = v[i + 2] < -32767 ? -32767 : v[i + 2], c3 = v[i + 3] < -32767 ? -32767 : v[i + 3];
        s0 += q[i] * ((float)c0 * INV32767);
        s1 += q[i + 1] * ((float)c1 * INV32767);
        s2 += q[i + 2] * ((float)c2 * INV32767);
        s3 += q[i + 3] * ((float)c3 * INV32767);
    }
    sum += ((s0 + s1) + s2) + s3;
    for (; i < dim; i++) {
        int16_t c = v[i] < -32767 ? -32767 : v[i];
        sum += q[i] * ((float)c * INV32767);
    }
    return sum;
}

/* dotFloat32 (index.go:198-214): dotFloat32AVX2 (dot_amd64.s:80-105, fused
 * lanes) on the dim&^7 prefix, unfused scalar tail. */
float orc_dot_f32_ref(const float *a, const float *b, int dim) {
    float sum = 0.0f;
    int start = 0;
    if (dim >= 8) {
        int n = dim & ~7;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < n; k += 8)
            for (int l = 0; l < 8; l++) acc[l] = fmaf(b[k + l], a[k + l], acc[l]);
        sum += hsum8(acc);
        start = n;
    }
    for (int i = start; i < dim; i++) sum += a[i] * b[i];
    return sum;
}

typedef struct { int idx; float dist; } cand_t;

static const int32_t *g_sort_ids;
static int cmp_cand(const void *pa, const void *pb) { /* index.go:141-146 */
    const cand_t *a = (const cand_t *)pa, *b = (const cand_t *)pb;
    if (a->dist == b->dist) {
        int32_t ia = g_sort_ids[a->idx], ib = g_sort_ids[b->idx];
        return ia < ib ? -1 : (ia > ib ? 1 : 0);
    }
    return a->dist > b->dist ? -1 : 1;
}

int orc_search_ref(int quant, const void *data, const int32_t *ids, int64_t count, int dim,
                   const float *query, int topK, int32_t *out_ids, float *out_dist) {
    if (topK > count) topK = (int)count;
    if (topK == 0) return 0;
    cand_t *best = (cand_t *)malloc(sizeof(cand_t) * (size_t)topK);
    int nb = 0, minIdx = -1;
    float minDist = 1.0f;
    for (int64_t i = 0; i < count; i++) {
        float dist;
        if (quant == 0) dist = orc_dot_f32_ref((const float *)data + i * dim, query, dim);
        else if (quant == 1) dist = orc_dot_int8_ref((const int8_t *)data + i * dim, query, dim);
        else dist = orc_dot_int16_ref((const int16_t *)data + i * dim, query, dim);
        if (nb < topK) {
            best[nb].idx = (int)i; best[nb].dist = dist; nb++;
            if (nb == topK) {
                minIdx = 0; minDist = best[0].dist;
                for (int k = 1; k < nb; k++) if (best[k].dist < minDist) { minDist = best[k].dist; minIdx = k; }
            }
            continue;
        }
        if (dist <= minDist) continue;
        best[minIdx].idx = (int)i; best[minIdx].dist = dist;
        minIdx = 0; minDist = best[0].dist;
        for (int k = 1; k < nb; k++) if (best[k].dist < minDist) { minDist = best[k].dist; minIdx = k; }
    }
    g_sort_ids = ids;
    qsort(best, (size_t)nb, sizeof(cand_t), cmp_cand);
    for (int k = 0; k < nb; k++) { out_ids[k] = ids[best[k].idx]; out_dist[k] = best[k].dist; }
    free(best);
    return nb;
}

/* Integer contract: exact int32 scores, total order (score desc, row asc). */
int orc_search_exact(int quant, const void *data, int64_t count, int dim, const void *qcodes,
                     int topk, int32_t *out_rows, int32_t *out_scores, float *out_dist) {
    if (topk > count) topk = (int)count;
    if (topk <= 0) return 0;
    int n = 0;
    for (int64_t r = 0; r < count; r++) {
        int32_t s = 0;
        if (quant == 1) {
            const int8_t *v = (const int8_t *)data + r * dim, *q = (const int8_t *)qcodes;
            for (int i = 0; i < dim; i++) s += (int32_t)q[i] * (int32_t)v[i];
        } else {
            const int16_t *v = (const int16_t *)data + r * dim, *q = (const int16_t *)qcodes;
            for (int i = 0; i < dim; i++) s += (int32_t)q[i] * (int32_t)v[i];
        }
        /* insertion into a sorted list: (score desc, row asc); rows arrive ascending */
        if (n == topk && s <= out_scores[n - 1]) continue;
        int p = n < topk ? n : topk - 1;
        while (p > 0 && out_scores[p - 1] < s) {
            out_scores[p] = out_scores[p - 1]; out_rows[p] = out_rows[p - 1]; p--;
        }
        out_scores[p] = s; out_rows[p] = (int32_t)r;
        if (n < topk) n++;
    }
    double sc2 = quant == 1 ? 127.0 * 127.0 : 32767.0 * 32767.0;
    for (int k = 0; k < n; k++) out_dist[k] = (float)((double)out_scores[k] / sc2);
    return n;
}

int orc_search_exact_batch(int quant, const void *data, int64_t count, int dim, const void *qcodes,
                           int nq, int topk, int32_t *out_rows, int32_t *out_scores, float *out_dist,
                           int nthreads) {
    int esz = quant == 1 ? 1 : 2;
    int kk = topk > count ? (int)count : topk;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    (void)nthreads;
#endif
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
    for (int qi = 0; qi < nq; qi++)
        orc_search_exact(quant, data, count, dim, (const uint8_t *)qcodes + (size_t)qi * dim * esz, topk,
                         out_rows + (size_t)qi * topk, out_scores + (size_t)qi * topk,
                         out_dist + (size_t)qi * topk);
    return kk;
}
