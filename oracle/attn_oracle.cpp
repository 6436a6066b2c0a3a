// attn_oracle.cpp - CPU restatement of GGML_OP_FLASH_ATTN_EXT for parity testing.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline / reference arm load this library, and only as the checker or the timed CPU
// baseline.  The product (libmm3fa.so) never links or calls it.
//
// Parity status: UNPINNED at the op boundary.  The reference's own implementation of this
// op lives in its ggml submodule (.gitmodules:1-3, github.com/ServeurpersoCom/ggml, pinned
// commit unknown), which is an empty directory in the mounted tree, so neither golden
// vectors nor a runnable reference exist.  This file restates the op from its mathematical
// contract as the reference's callers use it:
//   * tensor layouts, views and strides: src/qwen3-lm.h:400-439 (prefill), :784-824
//     (batched decode), src/dit.h:201-226 (DiT);
//   * semantics = the reference's own non-flash fallback, src/qwen3-enc.h:74-85
//     (mul_mat(k,q) -> soft_max_ext(scores, mask, scale) -> mul_mat(v^T, p) -> permute),
//     i.e. out = softmax(scale*q.k + mask) v with heads before rows in the result;
//   * masks as the host builds them: 0 / -inf, src/qwen3-lm.h:604-617 and :909-920.
// It is cross-checked against torch SDPA in float64 and, for Q8_0, against gguf-py 0.19.0's
// numpy codec (tests/test_oracle.py).
//
// Three modes:
//   ORC_EXACT    (0): double accumulation everywhere, Q used at full precision: ground truth.
//   ORC_F32ACC   (1): Q rounded to K's vec-dot type before the dot (F16/BF16 rounding, or
//                     Q8_0 quantization when K is Q8_0), F32 scores, one-pass F32 online
//                     softmax, F32 V accumulation: the precision the callers ask for with
//                     ggml_flash_attn_ext_set_prec(GGML_PREC_F32) (src/qwen3-lm.h:435,820,
//                     src/dit.h:222).  This is the parity bar of the GPU kernels.
//   ORC_GGML_CPU (2): ggml's CPU kernel as published in ggml-cpu (the one-row-at-a-time
//                     flash_attn_ext_f16 loop: Q converted to K's vec_dot_type, kq_vec_dot,
//                     expf online softmax), which keeps the V accumulator in F16 when V is F16
//                     (ggml_vec_mad_f16: y <- f16(y + v*p), ggml_vec_scale_f16 on a new
//                     maximum) and in F32 otherwise (V converted with to_float).  ggml-cpu
//                     ignores the F32 precision request, so this is what the reference's
//                     CPU backend would compute; with F16 V it is less accurate than
//                     ORC_F32ACC (one f16 rounding per key of the accumulated sum).
//
// Formats restated from their published definitions:
//   * IEEE 754 binary16 / bfloat16 conversions (round to nearest even);
//   * ggml Q8_0: blocks of 32 values = fp16 scale d + 32 int8 q, value = d*q; quantizer
//     d = max|x|/127, id = 1/d, q = roundf(x*id) (gguf-py quants.py Q8_0 follows the
//     same recipe);
//   * ALiBi slopes for max_bias > 0 (Press et al.; ggml's n_head_log2 split into m0/m1).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#if defined(__x86_64__)
#    include <immintrin.h>
#endif

extern "C" {

typedef struct orc_tensor {
    int32_t  type;
    int32_t  reserved;
    int64_t  ne[4];
    uint64_t nb[4];
    void *   data;
} orc_tensor;

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_BF16 = 30 };
enum { ORC_EXACT = 0, ORC_F32ACC = 1, ORC_GGML_CPU = 2 };
enum { QK8_0 = 32, Q8_0_BLOCK_BYTES = 34 };

// ---------------------------------------------------------------- scalar formats

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t exp  = (h >> 10) & 0x1fu;
    const uint32_t man  = h & 0x3ffu;
    uint32_t       bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: man * 2^-24, exact in binary32
            float f = (float) man * 5.9604644775390625e-8f;
            std::memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float out;
    std::memcpy(&out, &bits, 4);
    return out;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax   = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {  // inf / nan (nan keeps a quiet payload bit)
        return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) {  // >= 65520 rounds to inf
        return (uint16_t) (sign | 0x7c00u);
    }
    if (ax < 0x38800000u) {  // below 2^-14: subnormal half, value/2^-24 rounded to even
        float af;
        std::memcpy(&af, &ax, 4);
        const uint32_t m = (uint32_t) std::nearbyint(af * 16777216.0f);
        return (uint16_t) (sign | m);
    }
    const uint32_t e   = (ax >> 23) - 127 + 15;
    const uint32_t man = ax & 0x7fffffu;
    uint32_t       h   = (e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        h++;  // a carry out of the mantissa correctly bumps the exponent
    }
    return (uint16_t) (sign | h);
}

float orc_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t) b << 16;
    float    out;
    std::memcpy(&out, &bits, 4);
    return out;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) {
        return (uint16_t) ((x >> 16) | 0x40u);
    }
    const uint32_t lsb = (x >> 16) & 1u;
    return (uint16_t) ((x + 0x7fffu + lsb) >> 16);
}

// ---------------------------------------------------------------- Q8_0 codec

// Quantizes n (multiple of 32) floats into n/32 Q8_0 blocks.
void orc_q8_0_quantize_row(const float * x, uint8_t * out, int64_t n) {
    for (int64_t b = 0; b < n / QK8_0; b++) {
        const float * xb   = x + b * QK8_0;
        float         amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            amax = std::fmax(amax, std::fabs(xb[j]));
        }
        const float    d  = amax / 127.0f;
        const float    id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t *      ob = out + b * Q8_0_BLOCK_BYTES;
        const uint16_t dh = orc_f32_to_f16(d);
        std::memcpy(ob, &dh, 2);
        for (int j = 0; j < QK8_0; j++) {
            ob[2 + j] = (uint8_t) (int8_t) std::round(xb[j] * id);
        }
    }
}

void orc_q8_0_dequantize_row(const uint8_t * in, float * y, int64_t n) {
    for (int64_t b = 0; b < n / QK8_0; b++) {
        const uint8_t * ib = in + b * Q8_0_BLOCK_BYTES;
        uint16_t        dh;
        std::memcpy(&dh, ib, 2);
        const float d = orc_f16_to_f32(dh);
        for (int j = 0; j < QK8_0; j++) {
            y[b * QK8_0 + j] = d * (float) (int8_t) ib[2 + j];
        }
    }
}

// ---------------------------------------------------------------- row helpers

static float g_f16_table[65536];
static std::atomic<int> g_table_ready{ 0 };

static void init_tables() {
    if (g_table_ready.load(std::memory_order_acquire)) {
        return;
    }
    static std::atomic<int> once{ 0 };
    int                     expected = 0;
    if (once.compare_exchange_strong(expected, 1)) {
        for (uint32_t i = 0; i < 65536; i++) {
            g_f16_table[i] = orc_f16_to_f32((uint16_t) i);
        }
        g_table_ready.store(1, std::memory_order_release);
    } else {
        while (!g_table_ready.load(std::memory_order_acquire)) {
            std::this_thread::yield();
        }
    }
}

static inline const uint8_t * elem_ptr(const orc_tensor * t, int64_t i1, int64_t i2, int64_t i3) {
    return (const uint8_t *) t->data + i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3];
}

// Converts one row of n elements of any supported type to float.
static void row_to_f32(int type, const uint8_t * p, float * out, int64_t n) {
    switch (type) {
        case ORC_F32:
            std::memcpy(out, p, (size_t) n * 4);
            break;
        case ORC_F16:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                out[i] = g_f16_table[h];
            }
            break;
        case ORC_BF16:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                out[i] = orc_bf16_to_f32(h);
            }
            break;
        case ORC_Q8_0:
            orc_q8_0_dequantize_row(p, out, n);
            break;
        default:
            break;
    }
}

// ALiBi slope of query head h (slope 1 when max_bias == 0).
float orc_alibi_slope(int h, int n_head, float max_bias) {
    if (max_bias <= 0.0f) {
        return 1.0f;
    }
    const int   n_head_log2 = 1 << (int) std::floor(std::log2((double) n_head));
    const float m0          = std::pow(2.0f, -max_bias / (float) n_head_log2);
    const float m1          = std::pow(2.0f, -max_bias / 2.0f / (float) n_head_log2);
    return h < n_head_log2 ? std::pow(m0, (float) (h + 1)) : std::pow(m1, (float) (2 * (h - n_head_log2) + 1));
}

// ---------------------------------------------------------------- vector kernels

static inline float dot_f32(const float * a, const float * b, int64_t n) {
    float acc[8] = { 0, 0, 0, 0, 0, 0, 0, 0 };
    int64_t i    = 0;
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; l++) {
            acc[l] += a[i + l] * b[i + l];
        }
    }
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; i < n; i++) {
        s += a[i] * b[i];
    }
    return s;
}

// float64 dot of two float rows (four independent partial sums)
static inline double dot_f64_scalar(const float * a, const float * b, int64_t n) {
    double  acc[4] = { 0, 0, 0, 0 };
    int64_t i      = 0;
    for (; i + 4 <= n; i += 4) {
        for (int l = 0; l < 4; l++) {
            acc[l] += (double) a[i + l] * (double) b[i + l];
        }
    }
    double s = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    for (; i < n; i++) {
        s += (double) a[i] * (double) b[i];
    }
    return s;
}

static inline void axpy_f64_scalar(double * y, const float * x, double a, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        y[i] += a * (double) x[i];
    }
}

// One step of the F16 accumulator of ggml's CPU kernel (ggml_vec_mad_f16): y <- f16(y + x*v),
// the product and sum formed in F32 with one rounding (FMA), then rounded to F16.
static inline void mad_f16_scalar(uint16_t * y, const uint16_t * x, float v, int64_t n);
// ggml_vec_scale_f16: y <- f16(y * v)
static inline void scale_f16_scalar(uint16_t * y, float v, int64_t n);

#if defined(__x86_64__)
__attribute__((target("avx2,fma,f16c"))) static float dot_f32_f16_avx2(const float * a, const uint16_t * b,
                                                                          int64_t n) {
    __m256  acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    int64_t i    = 0;
    for (; i + 16 <= n; i += 16) {
        __m256 b0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (b + i)));
        __m256 b1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (b + i + 8)));
        acc0      = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), b0, acc0);
        acc1      = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), b1, acc1);
    }
    acc0     = _mm256_add_ps(acc0, acc1);
    __m128 s = _mm_add_ps(_mm256_castps256_ps128(acc0), _mm256_extractf128_ps(acc0, 1));
    s        = _mm_hadd_ps(s, s);
    s        = _mm_hadd_ps(s, s);
    float r  = _mm_cvtss_f32(s);
    for (; i < n; i++) {
        r += a[i] * g_f16_table[b[i]];
    }
    return r;
}

__attribute__((target("avx2,fma,f16c"))) static void axpy_f16_avx2(float * y, const uint16_t * x, float a,
                                                                     int64_t n) {
    const __m256 va = _mm256_set1_ps(a);
    int64_t      i  = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 xv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (x + i)));
        _mm256_storeu_ps(y + i, _mm256_fmadd_ps(va, xv, _mm256_loadu_ps(y + i)));
    }
    for (; i < n; i++) {
        y[i] += a * g_f16_table[x[i]];
    }
}

__attribute__((target("avx2,fma,f16c"))) static void mad_f16_avx2(uint16_t * y, const uint16_t * x, float v,
                                                                    int64_t n) {
    const __m256 vv = _mm256_set1_ps(v);
    int64_t      i  = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 xv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (x + i)));
        __m256 yv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (y + i)));
        yv        = _mm256_fmadd_ps(xv, vv, yv);
        _mm_storeu_si128((__m128i *) (y + i), _mm256_cvtps_ph(yv, _MM_FROUND_TO_NEAREST_INT));
    }
    mad_f16_scalar(y + i, x + i, v, n - i);
}

__attribute__((target("avx2,fma,f16c"))) static void scale_f16_avx2(uint16_t * y, float v, int64_t n) {
    const __m256 vv = _mm256_set1_ps(v);
    int64_t      i  = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 yv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (y + i)));
        _mm_storeu_si128((__m128i *) (y + i), _mm256_cvtps_ph(_mm256_mul_ps(yv, vv), _MM_FROUND_TO_NEAREST_INT));
    }
    scale_f16_scalar(y + i, v, n - i);
}

__attribute__((target("avx2,fma"))) static double dot_f64_avx2(const float * a, const float * b, int64_t n) {
    __m256d acc0 = _mm256_setzero_pd(), acc1 = _mm256_setzero_pd();
    int64_t i    = 0;
    for (; i + 8 <= n; i += 8) {
        acc0 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(a + i)), _mm256_cvtps_pd(_mm_loadu_ps(b + i)), acc0);
        acc1 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(a + i + 4)), _mm256_cvtps_pd(_mm_loadu_ps(b + i + 4)),
                               acc1);
    }
    acc0      = _mm256_add_pd(acc0, acc1);
    double t[4];
    _mm256_storeu_pd(t, acc0);
    double s = (t[0] + t[1]) + (t[2] + t[3]);
    for (; i < n; i++) {
        s += (double) a[i] * (double) b[i];
    }
    return s;
}

__attribute__((target("avx2,fma"))) static void axpy_f64_avx2(double * y, const float * x, double a, int64_t n) {
    const __m256d va = _mm256_set1_pd(a);
    int64_t       i  = 0;
    for (; i + 4 <= n; i += 4) {
        _mm256_storeu_pd(y + i, _mm256_fmadd_pd(va, _mm256_cvtps_pd(_mm_loadu_ps(x + i)), _mm256_loadu_pd(y + i)));
    }
    for (; i < n; i++) {
        y[i] += a * (double) x[i];
    }
}

static const bool g_has_avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
                               __builtin_cpu_supports("f16c");
#else
static const bool g_has_avx2 = false;
#endif

static inline void mad_f16_scalar(uint16_t * y, const uint16_t * x, float v, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        y[i] = orc_f32_to_f16(std::fmaf(g_f16_table[x[i]], v, g_f16_table[y[i]]));
    }
}

static inline void scale_f16_scalar(uint16_t * y, float v, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        y[i] = orc_f32_to_f16(g_f16_table[y[i]] * v);
    }
}

static inline void mad_f16(uint16_t * y, const uint16_t * x, float v, int64_t n) {
#if defined(__x86_64__)
    if (g_has_avx2) {
        mad_f16_avx2(y, x, v, n);
        return;
    }
#endif
    mad_f16_scalar(y, x, v, n);
}

static inline void scale_f16(uint16_t * y, float v, int64_t n) {
#if defined(__x86_64__)
    if (g_has_avx2) {
        scale_f16_avx2(y, v, n);
        return;
    }
#endif
    scale_f16_scalar(y, v, n);
}

static inline double dot_f64(const float * a, const float * b, int64_t n) {
#if defined(__x86_64__)
    if (g_has_avx2) {
        return dot_f64_avx2(a, b, n);
    }
#endif
    return dot_f64_scalar(a, b, n);
}

static inline void axpy_f64(double * y, const float * x, double a, int64_t n) {
#if defined(__x86_64__)
    if (g_has_avx2) {
        axpy_f64_avx2(y, x, a, n);
        return;
    }
#endif
    axpy_f64_scalar(y, x, a, n);
}

// Q8_0 x Q8_0 dot: per block int32 sum times the product of both fp16 scales.
static float dot_q8_0(const uint8_t * a, const uint8_t * b, int64_t n) {
    float s = 0.0f;
    for (int64_t blk = 0; blk < n / QK8_0; blk++) {
        const uint8_t * ab = a + blk * Q8_0_BLOCK_BYTES;
        const uint8_t * bb = b + blk * Q8_0_BLOCK_BYTES;
        int32_t         si = 0;
        for (int j = 0; j < QK8_0; j++) {
            si += (int32_t) (int8_t) ab[2 + j] * (int32_t) (int8_t) bb[2 + j];
        }
        uint16_t da, db;
        std::memcpy(&da, ab, 2);
        std::memcpy(&db, bb, 2);
        s += (float) si * (g_f16_table[da] * g_f16_table[db]);
    }
    return s;
}

// ---------------------------------------------------------------- the operator

struct orc_job {
    const orc_tensor *q, *k, *v, *mask;
    orc_tensor *      dst;
    float             scale, max_bias, softcap;
    int               mode;
};

static int64_t type_row_bytes(int type, int64_t n) {
    switch (type) {
        case ORC_F32:
            return 4 * n;
        case ORC_F16:
        case ORC_BF16:
            return 2 * n;
        case ORC_Q8_0:
            return n / QK8_0 * Q8_0_BLOCK_BYTES;
        default:
            return -1;
    }
}

// Per-thread scratch.  The exact mode converts the K and V slab of one (kv head, kv sequence)
// to float once and reuses it for every query row of that slab the thread takes.
struct orc_scratch {
    std::vector<float>    qf, kf, vf, accf;
    std::vector<double>   accd, sc;
    std::vector<uint8_t>  qq;
    std::vector<uint16_t> q16, acc16;
    std::vector<float>    kslab, vslab;
    int64_t               slab_kh = -1, slab_ks = -1;
};

static void load_slab(const orc_job & J, int64_t kh, int64_t ks, orc_scratch & W) {
    if (W.slab_kh == kh && W.slab_ks == ks) {
        return;
    }
    const int64_t D = J.k->ne[0], DV = J.v->ne[0], n_kv = J.k->ne[1];
    W.kslab.resize((size_t) (n_kv * D));
    W.vslab.resize((size_t) (n_kv * DV));
    for (int64_t j = 0; j < n_kv; j++) {
        row_to_f32(J.k->type, elem_ptr(J.k, j, kh, ks), W.kslab.data() + j * D, D);
        row_to_f32(J.v->type, elem_ptr(J.v, j, kh, ks), W.vslab.data() + j * DV, DV);
    }
    W.slab_kh = kh;
    W.slab_ks = ks;
}

// One query row (i, h, s) of the operator.
static void run_row(const orc_job & J, int64_t i, int64_t h, int64_t s, orc_scratch & W) {
    const orc_tensor *q = J.q, *k = J.k, *v = J.v, *mask = J.mask;
    const int64_t     D = q->ne[0], DV = v->ne[0], n_kv = k->ne[1];
    const int64_t     n_head = q->ne[2];
    const int64_t     kh     = h / (q->ne[2] / k->ne[2]);
    const int64_t     ks     = s / (q->ne[3] / k->ne[3]);
    const float       slope  = orc_alibi_slope((int) h, (int) n_head, J.max_bias);
    float *           qf     = W.qf.data();

    row_to_f32(q->type, elem_ptr(q, i, h, s), qf, D);
    const uint8_t * mrow = nullptr;
    if (mask) {
        mrow = (const uint8_t *) mask->data + i * mask->nb[1] + (h % mask->ne[2]) * mask->nb[2] +
               (s % mask->ne[3]) * mask->nb[3];
    }
    auto mask_at = [&](int64_t j) -> float {
        if (!mrow) {
            return 0.0f;
        }
        if (mask->type == ORC_F32) {
            float m;
            std::memcpy(&m, mrow + 4 * j, 4);
            return m;
        }
        uint16_t m;
        std::memcpy(&m, mrow + 2 * j, 2);
        return g_f16_table[m];
    };
    float *dst_row = (float *) ((uint8_t *) J.dst->data + h * J.dst->nb[1] + i * J.dst->nb[2] + s * J.dst->nb[3]);

    if (J.mode == ORC_EXACT) {
        // two-pass softmax in double over the float slab: scores, max, exp-sum, weighted V
        load_slab(J, kh, ks, W);
        double * sc = W.sc.data();
        double   mx = -INFINITY;
        for (int64_t j = 0; j < n_kv; j++) {
            const float mv = mask_at(j);
            if (mv == -INFINITY) {
                sc[j] = -INFINITY;
                continue;
            }
            double sv = dot_f64(qf, W.kslab.data() + j * D, D) * (double) J.scale;
            if (J.softcap != 0.0f) {
                sv = (double) J.softcap * std::tanh(sv / (double) J.softcap);
            }
            sv += (double) slope * (double) mv;
            sc[j] = sv;
            if (sv > mx) {
                mx = sv;
            }
        }
        double * accd = W.accd.data();
        std::fill(accd, accd + DV, 0.0);
        double sum = 0.0;
        if (mx != -INFINITY) {
            for (int64_t j = 0; j < n_kv; j++) {
                if (sc[j] == -INFINITY) {
                    continue;
                }
                const double p = std::exp(sc[j] - mx);
                sum += p;
                axpy_f64(accd, W.vslab.data() + j * DV, p, DV);
            }
        }
        for (int64_t d = 0; d < DV; d++) {
            dst_row[d] = sum > 0.0 ? (float) (accd[d] / sum) : 0.0f;
        }
        return;
    }

    // F32ACC and GGML_CPU: Q rounded to K's vec-dot type, F32 scores, one-pass online softmax.
    const bool  acc16     = J.mode == ORC_GGML_CPU && v->type == ORC_F16;
    const float scale_eff = J.softcap != 0.0f ? J.scale / J.softcap : J.scale;
    if (k->type == ORC_F16) {
        for (int64_t d = 0; d < D; d++) {
            W.q16[(size_t) d] = orc_f32_to_f16(qf[d]);
            qf[d]             = g_f16_table[W.q16[(size_t) d]];
        }
    } else if (k->type == ORC_BF16) {
        for (int64_t d = 0; d < D; d++) {
            qf[d] = orc_bf16_to_f32(orc_f32_to_bf16(qf[d]));
        }
    } else if (k->type == ORC_Q8_0) {
        orc_q8_0_quantize_row(qf, W.qq.data(), D);
    }
    float *    accf = W.accf.data();
    uint16_t * a16  = W.acc16.data();
    std::fill(accf, accf + DV, 0.0f);
    std::fill(a16, a16 + DV, (uint16_t) 0);
    float M = -INFINITY, S = 0.0f;
    for (int64_t j = 0; j < n_kv; j++) {
        const float mv = mask_at(j);
        if (mv == -INFINITY) {
            continue;  // contributes exp(-inf) = 0
        }
        const uint8_t * kp = elem_ptr(k, j, kh, ks);
        float           dot;
        if (k->type == ORC_Q8_0) {
            dot = dot_q8_0(W.qq.data(), kp, D);
        } else if (k->type == ORC_F16 && g_has_avx2) {
#if defined(__x86_64__)
            dot = dot_f32_f16_avx2(qf, (const uint16_t *) kp, D);
#else
            dot = 0.0f;
#endif
        } else {
            row_to_f32(k->type, kp, W.kf.data(), D);
            dot = dot_f32(qf, W.kf.data(), D);
        }
        float sv = dot * scale_eff;
        if (J.softcap != 0.0f) {
            sv = J.softcap * std::tanh(sv);
        }
        sv += slope * mv;
        if (sv == -INFINITY) {
            continue;
        }
        float ms = 1.0f, vs = 1.0f;
        if (sv > M) {
            ms = M == -INFINITY ? 0.0f : std::exp(M - sv);
            M  = sv;
            if (acc16) {
                scale_f16(a16, ms, DV);
            } else if (ms != 1.0f) {
                for (int64_t d = 0; d < DV; d++) {
                    accf[d] *= ms;
                }
            }
        } else {
            vs = std::exp(sv - M);
        }
        const uint8_t * vp = elem_ptr(v, j, kh, ks);
        if (acc16) {
            mad_f16(a16, (const uint16_t *) vp, vs, DV);
        } else if (v->type == ORC_F16 && g_has_avx2) {
#if defined(__x86_64__)
            axpy_f16_avx2(accf, (const uint16_t *) vp, vs, DV);
#endif
        } else {
            row_to_f32(v->type, vp, W.vf.data(), DV);
            for (int64_t d = 0; d < DV; d++) {
                accf[d] += vs * W.vf[(size_t) d];
            }
        }
        S = S * ms + vs;
    }
    if (acc16) {
        for (int64_t d = 0; d < DV; d++) {
            accf[d] = g_f16_table[a16[d]];
        }
    }
    const float inv = S > 0.0f ? 1.0f / S : 0.0f;
    for (int64_t d = 0; d < DV; d++) {
        dst_row[d] = accf[d] * inv;
    }
}

// Returns 0 on success, a positive code on malformed operands.
int orc_flash_attn_ext(const orc_tensor * q, const orc_tensor * k, const orc_tensor * v, const orc_tensor * mask,
                       float scale, float max_bias, float logit_softcap, int mode, orc_tensor * dst, int n_threads) {
    init_tables();
    if (!q || !k || !v || !dst) {
        return 1;
    }
    if (mode != ORC_EXACT && mode != ORC_F32ACC && mode != ORC_GGML_CPU) {
        return 4;
    }
    if (q->ne[0] != k->ne[0] || k->ne[1] != v->ne[1] || k->ne[2] != v->ne[2] || k->ne[3] != v->ne[3]) {
        return 3;
    }
    if (q->ne[2] % k->ne[2] != 0 || q->ne[3] % k->ne[3] != 0) {
        return 3;
    }
    if (dst->ne[0] != v->ne[0] || dst->ne[1] != q->ne[2] || dst->ne[2] != q->ne[1] || dst->ne[3] != q->ne[3]) {
        return 3;
    }
    if (mask && (mask->ne[0] != k->ne[1] || mask->ne[1] < q->ne[1] || q->ne[2] % mask->ne[2] != 0 ||
                 q->ne[3] % mask->ne[3] != 0)) {
        return 3;
    }
    if (type_row_bytes(k->type, k->ne[0]) < 0 || type_row_bytes(v->type, v->ne[0]) < 0 ||
        type_row_bytes(q->type, q->ne[0]) < 0) {
        return 2;
    }
    orc_job J{ q, k, v, mask, dst, scale, max_bias, logit_softcap, mode };

    const int64_t n_rows = q->ne[1] * q->ne[2] * q->ne[3];
    if (n_threads < 1) {
        n_threads = 1;
    }
    if ((int64_t) n_threads > n_rows) {
        n_threads = (int) std::max<int64_t>(n_rows, 1);
    }
    // rows are handed out in chunks of consecutive rows (i fastest, then h, then s), so a
    // thread's rows mostly share one (kv head, kv sequence) slab
    const int64_t        chunk = std::max<int64_t>(1, std::min<int64_t>(64, n_rows / ((int64_t) n_threads * 8)));
    std::atomic<int64_t> next{ 0 };
    auto                 worker = [&]() {
        const int64_t D = q->ne[0], DV = v->ne[0];
        orc_scratch   W;
        W.qf.resize((size_t) D);
        W.kf.resize((size_t) D);
        W.vf.resize((size_t) DV);
        W.accf.resize((size_t) DV);
        W.accd.resize((size_t) DV);
        W.acc16.resize((size_t) DV);
        W.sc.resize((size_t) std::max<int64_t>(k->ne[1], 1));
        W.qq.resize((size_t) (D / QK8_0 + 1) * Q8_0_BLOCK_BYTES);
        W.q16.resize((size_t) D);
        for (;;) {
            const int64_t r0 = next.fetch_add(chunk);
            if (r0 >= n_rows) {
                break;
            }
            for (int64_t r = r0; r < std::min(n_rows, r0 + chunk); r++) {
                const int64_t i = r % q->ne[1];
                const int64_t h = (r / q->ne[1]) % q->ne[2];
                const int64_t s = r / (q->ne[1] * q->ne[2]);
                run_row(J, i, h, s, W);
            }
        }
    };
    if (n_threads == 1) {
        worker();
    } else {
        std::vector<std::thread> th;
        th.reserve((size_t) n_threads);
        for (int t = 0; t < n_threads; t++) {
            th.emplace_back(worker);
        }
        for (auto & t : th) {
            t.join();
        }
    }
    return 0;
}

// Vectorised helpers for the Python side (tests build fixtures through these).
void orc_f32_to_f16_array(const float * x, uint16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        y[i] = orc_f32_to_f16(x[i]);
    }
}

void orc_f16_to_f32_array(const uint16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        y[i] = orc_f16_to_f32(x[i]);
    }
}

int orc_version(void) {
    return 1;
}

}  // extern "C"
