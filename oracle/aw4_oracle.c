/*
 * aw4_oracle.c -- CPU restatement of the reference 4-bit AdamW step.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (adamw4bit_b200/) links,
 * loads or calls this file.  It is used by tests/, by __graft_entry__.smoke()
 * as the checker, and by bench.py's cpu_baseline / --impl reference leg as the
 * timed CPU implementation.  It restates, in plain C with IEEE float32
 * arithmetic, the algorithm of nubank/adamw4bit:
 *
 *   src/adamw4bit/adamw.py          QuantizedAdamW.step   (lines 472-805)
 *   src/adamw4bit/quantization.py   _quantize_impl        (lines 898-971)
 *                                   dequantize            (lines 975-1004)
 *                                   strategies            (lines 240-377, 529-552)
 *                                   nibble packing        (lines 627-691)
 *
 * Floating-point recipe (each item pinned against the reference's own CPU
 * output by tests/test_oracle_golden.py):
 *   - Tensor.lerp_(end, w) with |w| < 0.5 is fmaf(w, end - self, self)
 *     (torch ATen lerp formula; the CPU vector path uses a fused multiply-add).
 *   - tensor / python float is an IEEE float32 division by (float)scalar.
 *   - addcdiv_(t1, t2, value=v) is self + ((float)v * t1) / t2, no FMA.
 *   - 1.0 / t is an IEEE float32 reciprocal.
 *   - block sums over 128 values follow torch's CPU reduction order:
 *     8-lane vectors, 4 round-robin accumulators, lanes summed in order.
 *   - sqrt is IEEE sqrtf.  The reference's CPU sqrt goes through MKL VML for
 *     tensors of >= ~1024 elements and is not correctly rounded (1 ulp on
 *     ~0.7% of elements); that is the one op this oracle does not reproduce.
 *     It never reaches ZE-EDEN codes or scales (moments do not depend on the
 *     denominator); it perturbs parameters by ~1e-7 relative.
 *
 * The counter-based Philox4x32-10 generator (Salmon, Moraes, Dror, Shaw,
 * "Parallel random numbers: as easy as 1, 2, 3", SC'11) is restated here with
 * the counter layout the product kernel uses, so SR codes under Philox can be
 * compared bit-for-bit with the GPU as well.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off, no fast-math, OpenMP).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define AW4O_BLOCK 128

enum { AW4O_RTN = 0, AW4O_SR_VALUE = 1, AW4O_SR_UPDATE = 2 };
enum { AW4O_F32 = 0, AW4O_BF16 = 1, AW4O_F16 = 2 };

/* ------------------------------------------------------------------------ */
/* dtype conversions (c10::BFloat16 / c10::Half round-to-nearest-even)       */
/* ------------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }
static inline uint16_t f32_to_bf16(float f) {
    if (isnan(f)) return 0x7FC0;
    uint32_t u = f2u(f);
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7FFFu + lsb) >> 16);
}
static inline float f16_to_f32(uint16_t h) { _Float16 v; memcpy(&v, &h, 2); return (float)v; }
static inline uint16_t f32_to_f16(float f) { _Float16 v = (_Float16)f; uint16_t h; memcpy(&h, &v, 2); return h; }

static inline float load_elem(const void* base, int dtype, int64_t i) {
    switch (dtype) {
    case AW4O_BF16: return bf16_to_f32(((const uint16_t*)base)[i]);
    case AW4O_F16: return f16_to_f32(((const uint16_t*)base)[i]);
    default: return ((const float*)base)[i];
    }
}
static inline float round_elem(int dtype, float v) {
    /* Value after storing into a tensor of `dtype` and reading it back. */
    switch (dtype) {
    case AW4O_BF16: return bf16_to_f32(f32_to_bf16(v));
    case AW4O_F16: return f16_to_f32(f32_to_f16(v));
    default: return v;
    }
}
static inline void store_elem(void* base, int dtype, int64_t i, float v) {
    switch (dtype) {
    case AW4O_BF16: ((uint16_t*)base)[i] = f32_to_bf16(v); break;
    case AW4O_F16: ((uint16_t*)base)[i] = f32_to_f16(v); break;
    default: ((float*)base)[i] = v;
    }
}

/* ------------------------------------------------------------------------ */
/* Codebook rounding (quantization.py:254-377)                               */
/* ------------------------------------------------------------------------ */

/* torch.searchsorted(cb, x) (side='left'): first index i with cb[i] >= x.
 * ATen's lower-bound loop advances while !(cb[mid] >= x), so NaN maps to 16. */
static inline int searchsorted_left(const float* cb, float x) {
    int start = 0, end = 16;
    while (start < end) {
        int mid = start + ((end - start) >> 1);
        if (!(cb[mid] >= x)) start = mid + 1; else end = mid;
    }
    return start;
}

/* _CodebookQuantizationStrategy.quantize (quantization.py:254-272):
 * nearest of the two neighbours, ties round up. */
static inline int rtn_code(const float* cb, float x) {
    int i = searchsorted_left(cb, x);
    int left = i - 1 < 0 ? 0 : i - 1;
    int right = i > 15 ? 15 : i;
    float dl = fabsf(x - cb[left]);
    float dr = fabsf(cb[right] - x);
    return (dl < dr) ? left : right;
}

/* _StochasticCodebookQuantizationStrategy.quantize (quantization.py:286-315). */
static inline int value_sr_code(const float* cb, float x, float u) {
    int i = searchsorted_left(cb, x);
    int left = i - 1 < 0 ? 0 : i - 1;
    int right = i > 15 ? 15 : i;
    float a = cb[left], b = cb[right];
    float width = b - a;
    float wc = width < 1e-12f ? 1e-12f : width;          /* clamp_min(1e-12) */
    if (isnan(width)) wc = width;
    float p = (x - a) / wc;
    if (!(width > 0.0f)) p = 0.0f;                          /* where(width > 0, p, 0) */
    /* clamp_(0, 1) propagates NaN */
    if (p < 0.0f) p = 0.0f;
    if (p > 1.0f) p = 1.0f;
    return (u < p) ? right : left;
}

/* preconditioner(levels) of _UpdateUnbiasedStochasticCodebookQuantizationStrategy
 * (quantization.py:356-358): 1 / (sqrt(clamp_min(s * l / bias, 0)) + eps). */
static inline float precond(float s, float level, float bias_f, float eps_f) {
    float v = (s * level) / bias_f;
    if (v < 0.0f) v = 0.0f;                                  /* clamp_min(0.0); NaN stays */
    return 1.0f / (sqrtf(v) + eps_f);
}

/* quantization.py:327-377 */
static inline int update_sr_code(const float* cb, float x, float s, float bias_f,
                                 float eps_f, float u) {
    int i = searchsorted_left(cb, x);
    int left = i - 1 < 0 ? 0 : i - 1;
    int right = i > 15 ? 15 : i;
    float a = cb[left], b = cb[right];
    float width = b - a;
    float fl = precond(s, a, bias_f, eps_f);
    float fr = precond(s, b, bias_f, eps_f);
    float fx = precond(s, x, bias_f, eps_f);
    float den = fl - fr;
    float denc = den < 1e-30f ? 1e-30f : den;               /* clamp_min(1e-30) */
    if (isnan(den)) denc = den;
    float p = (fx - fr) / denc;
    if (!((width > 0.0f) && (den > 0.0f))) p = 1.0f;
    if (p < 0.0f) p = 0.0f;
    if (p > 1.0f) p = 1.0f;
    return (u < p) ? left : right;
}

/* Sum of 128 float32 values in torch's CPU reduction order for
 * (nb, 128).sum(dim=1): vector v (elements 8v..8v+7) accumulates into
 * accumulator v % 4, the four accumulators are combined in order, then the
 * eight lanes are summed in order starting from zero. */
static float torch_row_sum128(const float* v) {
    float acc[4][8];
    for (int k = 0; k < 4; ++k)
        for (int j = 0; j < 8; ++j) acc[k][j] = 0.0f;
    for (int vi = 0; vi < 16; ++vi)
        for (int j = 0; j < 8; ++j) acc[vi & 3][j] = acc[vi & 3][j] + v[8 * vi + j];
    float t[8];
    for (int j = 0; j < 8; ++j) t[j] = ((acc[0][j] + acc[1][j]) + acc[2][j]) + acc[3][j];
    float total = 0.0f;
    for (int j = 0; j < 8; ++j) total = total + t[j];
    return total;
}

/* torch.max propagates NaN; clamp(min=c) propagates NaN. */
static inline float nanmax(float a, float b) {
    if (isnan(a) || isnan(b)) return NAN;
    return a > b ? a : b;
}
static inline float clamp_min_nan(float a, float c) {
    if (isnan(a)) return a;
    return a < c ? c : a;
}

/* ------------------------------------------------------------------------ */
/* Philox4x32-10 (Salmon et al., SC'11)                                     */
/* ------------------------------------------------------------------------ */
static inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c[1] ^ k0;
        uint32_t n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
}

/* Uniform float in [0, 1) for element `e` of a tensor: counter
 * (e/4 low, e/4 high, step, ordinal), key = 64-bit stream key; word e%4,
 * top 24 bits.  Same layout as the product kernel. */
float aw4o_philox_uniform(uint64_t key, uint32_t step, uint32_t ordinal, uint64_t e) {
    uint64_t q = e >> 2;
    uint32_t c[4] = {(uint32_t)q, (uint32_t)(q >> 32), step, ordinal};
    philox4x32_10(c, (uint32_t)key, (uint32_t)(key >> 32));
    return (float)(c[e & 3] >> 8) * 0x1p-24f;
}

/* ------------------------------------------------------------------------ */
/* Block codec (quantization.py:898-1004)                                    */
/* ------------------------------------------------------------------------ */

typedef struct {
    const float* cb;      /* 16 sorted levels */
    int round_mode;       /* AW4O_RTN / AW4O_SR_VALUE / AW4O_SR_UPDATE */
    int zero_floor;       /* dyn4_nz: code 0 -> 1 (quantization.py:529-552) */
    int eden;             /* EDEN block-scale calibration (quantization.py:955-960) */
    float bias_f;         /* (float)max(bias_correction, 1e-12)  (update SR) */
    float eps_f;          /* (float)eps                          (update SR) */
} aw4o_codec;

/* One 128-value block: absmax scale (clamped at 1e-12), normalise, round,
 * optional EDEN.  `u` holds the 128 uniforms for SR modes (may be NULL for RTN). */
static void quantize_block(const aw4o_codec* q, const float* x, const float* u,
                           uint8_t* codes, float* scale_out) {
    float amax = 0.0f;
    for (int j = 0; j < AW4O_BLOCK; ++j) amax = nanmax(amax, fabsf(x[j]));
    float s = clamp_min_nan(amax, 1e-12f);
    float xs[AW4O_BLOCK];
    for (int j = 0; j < AW4O_BLOCK; ++j) {
        xs[j] = x[j] / s;
        int c;
        if (q->round_mode == AW4O_RTN) c = rtn_code(q->cb, xs[j]);
        else if (q->round_mode == AW4O_SR_VALUE) c = value_sr_code(q->cb, xs[j], u[j]);
        else c = update_sr_code(q->cb, xs[j], s, q->bias_f, q->eps_f, u[j]);
        if (q->zero_floor && c == 0) c = 1;
        codes[j] = (uint8_t)c;
    }
    if (q->eden) {
        float num[AW4O_BLOCK], den[AW4O_BLOCK];
        for (int j = 0; j < AW4O_BLOCK; ++j) {
            num[j] = xs[j] * xs[j];
            den[j] = xs[j] * q->cb[codes[j]];
        }
        float n = torch_row_sum128(num);
        float d = torch_row_sum128(den);
        float corr = n / clamp_min_nan(d, 1e-12f);
        s = s * corr;
    }
    *scale_out = s;
}

/* Public codec entry points used by tests (codes unpacked, one per byte). */
int aw4o_quantize(const float* x, int64_t n, const float* cb, int round_mode, int zero_floor,
                  int eden, const float* draws, double bias_correction, double eps,
                  uint8_t* codes, float* scales) {
    if (n % AW4O_BLOCK) return -1;
    aw4o_codec q = {cb, round_mode, zero_floor, eden,
                    (float)(bias_correction < 1e-12 ? 1e-12 : bias_correction), (float)eps};
    int64_t nb = n / AW4O_BLOCK;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b)
        quantize_block(&q, x + b * AW4O_BLOCK, draws ? draws + b * AW4O_BLOCK : NULL,
                       codes + b * AW4O_BLOCK, scales + b);
    return 0;
}

/* dequantize (quantization.py:975-1004): cb[code] * absmax[block]. */
void aw4o_dequantize(const uint8_t* codes, const float* scales, int64_t n, const float* cb,
                     float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = cb[codes[i] & 15] * scales[i / AW4O_BLOCK];
}

/* pack_4bit_codes (quantization.py:627-638): even element in the low nibble. */
void aw4o_pack(const uint8_t* codes, int64_t n, uint8_t* packed) {
    for (int64_t k = 0; k < (n + 1) / 2; ++k) {
        uint8_t lo = codes[2 * k];
        uint8_t hi = (2 * k + 1 < n) ? codes[2 * k + 1] : 0;
        packed[k] = (uint8_t)(lo | (uint8_t)(hi << 4));
    }
}

/* unpack_4bit_codes (quantization.py:641-654). */
void aw4o_unpack(const uint8_t* packed, int64_t n, uint8_t* codes) {
    for (int64_t i = 0; i < n; ++i) codes[i] = (packed[i >> 1] >> ((i & 1) * 4)) & 15;
}

/* ------------------------------------------------------------------------ */
/* Optimizer step (adamw.py:472-805)                                         */
/* ------------------------------------------------------------------------ */

typedef struct {
    int param_dtype, grad_dtype;     /* AW4O_F32 / AW4O_BF16 / AW4O_F16 */
    int m1_mode;                     /* AW4O_RTN or AW4O_SR_VALUE */
    int m2_mode;                     /* AW4O_RTN, AW4O_SR_VALUE or AW4O_SR_UPDATE */
    int m2_zero_floor, eden;
    int m2_next_bias;                /* dyn4_lookahead_sr: storage bias uses step t+1 */
    const float* cb1;
    const float* cb2;
    double lr, beta1, beta2, eps, weight_decay;
    int64_t step;                    /* t, already incremented (adamw.py:547) */
    /* Philox keys used when the matching draws pointer is NULL. */
    uint64_t m1_key, m2_key;
    uint32_t ordinal;
    int64_t elem_offset;             /* index of element 0 within the logical tensor */
} aw4o_step_cfg;

/* Host scalars, as the reference derives them in float64 and torch casts
 * them to float32 when they meet a float32 tensor (adamw.py:557-564,
 * 684-691, 743). */
typedef struct {
    float w1, w2, decay, neg_step, sqrt_bc2, eps, sr_bias;
} aw4o_scalars;

static aw4o_scalars make_scalars(const aw4o_step_cfg* c) {
    aw4o_scalars s;
    double bc1 = 1.0 - pow(c->beta1, (double)c->step);
    double bc2 = 1.0 - pow(c->beta2, (double)c->step);
    double step_size = c->lr / bc1;
    s.w1 = (float)(1.0 - c->beta1);
    s.w2 = (float)(1.0 - c->beta2);
    s.decay = (float)(1.0 - c->lr * c->weight_decay);
    s.neg_step = (float)(-step_size);
    s.sqrt_bc2 = (float)sqrt(bc2);
    s.eps = (float)c->eps;
    double storage_bc = c->m2_next_bias ? 1.0 - pow(c->beta2, (double)(c->step + 1)) : bc2;
    s.sr_bias = (float)(storage_bc < 1e-12 ? 1e-12 : storage_bc);
    return s;
}

/* Element update shared by the quantized and FP32-state paths:
 * m1.lerp_(g, 1-b1); m2.lerp_(g*g, 1-b2); den = sqrt(m2)/sqrt(bc2) + eps;
 * p *= 1-lr*wd; p += (-lr/bc1 * m1) / den. */
static inline void adamw_elem(const aw4o_scalars* s, int pdt, float g, float* m1, float* m2,
                              float* p) {
    *m1 = fmaf(s->w1, g - *m1, *m1);
    float gsq = g * g;
    *m2 = fmaf(s->w2, gsq - *m2, *m2);
    float den = sqrtf(*m2) / s->sqrt_bc2 + s->eps;
    float pv = round_elem(pdt, *p * s->decay);
    float upd = (s->neg_step * *m1) / den;
    *p = round_elem(pdt, pv + upd);
}

/* Step of one tensor with quantized m1/m2 (packed codes, per-block scales).
 * n must be a multiple of 128.  Draw pointers may be NULL, in which case the
 * Philox stream (cfg keys, step, ordinal, element index) supplies uniforms. */
int aw4o_step(const aw4o_step_cfg* c, void* param, const void* grad, int64_t n,
              uint8_t* m1_packed, float* m1_scales, uint8_t* m2_packed, float* m2_scales,
              const float* m1_draws, const float* m2_draws) {
    if (n % AW4O_BLOCK) return -1;
    aw4o_scalars s = make_scalars(c);
    aw4o_codec q1 = {c->cb1, c->m1_mode, 0, 0, s.sr_bias, s.eps};
    aw4o_codec q2 = {c->cb2, c->m2_mode, c->m2_zero_floor, c->eden, s.sr_bias, s.eps};
    int64_t nb = n / AW4O_BLOCK;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        float m1[AW4O_BLOCK], m2[AW4O_BLOCK], u1[AW4O_BLOCK], u2[AW4O_BLOCK];
        uint8_t c1[AW4O_BLOCK], c2[AW4O_BLOCK];
        int64_t base = b * AW4O_BLOCK;
        float s1 = m1_scales[b], s2 = m2_scales[b];
        for (int j = 0; j < AW4O_BLOCK; ++j) {
            int64_t i = base + j;
            uint8_t byte1 = m1_packed[i >> 1], byte2 = m2_packed[i >> 1];
            int k1 = (byte1 >> ((i & 1) * 4)) & 15, k2 = (byte2 >> ((i & 1) * 4)) & 15;
            m1[j] = c->cb1[k1] * s1;      /* dequantize (quantization.py:999) */
            m2[j] = c->cb2[k2] * s2;
            float g = load_elem(grad, c->grad_dtype, i);
            float p = load_elem(param, c->param_dtype, i);
            adamw_elem(&s, c->param_dtype, g, &m1[j], &m2[j], &p);
            store_elem(param, c->param_dtype, i, p);
        }
        if (c->m1_mode != AW4O_RTN)
            for (int j = 0; j < AW4O_BLOCK; ++j)
                u1[j] = m1_draws ? m1_draws[base + j]
                                 : aw4o_philox_uniform(c->m1_key, (uint32_t)c->step, c->ordinal,
                                                       (uint64_t)(c->elem_offset + base + j));
        if (c->m2_mode != AW4O_RTN)
            for (int j = 0; j < AW4O_BLOCK; ++j)
                u2[j] = m2_draws ? m2_draws[base + j]
                                 : aw4o_philox_uniform(c->m2_key, (uint32_t)c->step, c->ordinal,
                                                       (uint64_t)(c->elem_offset + base + j));
        quantize_block(&q1, m1, u1, c1, &m1_scales[b]);
        quantize_block(&q2, m2, u2, c2, &m2_scales[b]);
        for (int j = 0; j < AW4O_BLOCK; j += 2) {
            m1_packed[(base + j) >> 1] = (uint8_t)(c1[j] | (c1[j + 1] << 4));
            m2_packed[(base + j) >> 1] = (uint8_t)(c2[j] | (c2[j + 1] << 4));
        }
    }
    return 0;
}

/* Step of one tensor with an FP32 first moment next to a quantized second
 * moment (m1_quant_scheme="fp32": adamw.py:510-521 resolves each moment's
 * scheme separately, and an FP32 moment is a plain float32 tensor,
 * adamw.py:830-833).  m1 is updated in place; m2 is decoded, updated and
 * re-encoded exactly as in aw4o_step.  cfg->cb1 and m1_mode are unused. */
int aw4o_step_fp32_m1(const aw4o_step_cfg* c, void* param, const void* grad, int64_t n,
                      float* m1, uint8_t* m2_packed, float* m2_scales, const float* m2_draws) {
    if (n % AW4O_BLOCK) return -1;
    aw4o_scalars s = make_scalars(c);
    aw4o_codec q2 = {c->cb2, c->m2_mode, c->m2_zero_floor, c->eden, s.sr_bias, s.eps};
    int64_t nb = n / AW4O_BLOCK;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        float m2[AW4O_BLOCK], u2[AW4O_BLOCK];
        uint8_t c2[AW4O_BLOCK];
        int64_t base = b * AW4O_BLOCK;
        float s2 = m2_scales[b];
        for (int j = 0; j < AW4O_BLOCK; ++j) {
            int64_t i = base + j;
            int k2 = (m2_packed[i >> 1] >> ((i & 1) * 4)) & 15;
            m2[j] = c->cb2[k2] * s2;      /* dequantize (quantization.py:999) */
            float g = load_elem(grad, c->grad_dtype, i);
            float p = load_elem(param, c->param_dtype, i);
            adamw_elem(&s, c->param_dtype, g, &m1[i], &m2[j], &p);
            store_elem(param, c->param_dtype, i, p);
        }
        if (c->m2_mode != AW4O_RTN)
            for (int j = 0; j < AW4O_BLOCK; ++j)
                u2[j] = m2_draws ? m2_draws[base + j]
                                 : aw4o_philox_uniform(c->m2_key, (uint32_t)c->step, c->ordinal,
                                                       (uint64_t)(c->elem_offset + base + j));
        quantize_block(&q2, m2, u2, c2, &m2_scales[b]);
        for (int j = 0; j < AW4O_BLOCK; j += 2)
            m2_packed[(base + j) >> 1] = (uint8_t)(c2[j] | (c2[j + 1] << 4));
    }
    return 0;
}

/* Step of one tensor whose moments stay FP32 because it is not eligible for
 * quantized state (adamw.py:807-817: numel < 4096 or not a block multiple). */
int aw4o_step_fp32_state(const aw4o_step_cfg* c, void* param, const void* grad, int64_t n,
                         float* m1, float* m2) {
    aw4o_scalars s = make_scalars(c);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float g = load_elem(grad, c->grad_dtype, i);
        float p = load_elem(param, c->param_dtype, i);
        adamw_elem(&s, c->param_dtype, g, &m1[i], &m2[i], &p);
        store_elem(param, c->param_dtype, i, p);
    }
    return 0;
}

/* State initialisation (adamw.py:524-545): quantize a zero moment. */
int aw4o_init_zero(const float* cb, int round_mode, int zero_floor, int eden, int64_t n,
                   uint8_t* packed, float* scales) {
    if (n % AW4O_BLOCK) return -1;
    float zeros[AW4O_BLOCK] = {0};
    float u[AW4O_BLOCK];
    for (int j = 0; j < AW4O_BLOCK; ++j) u[j] = 0.5f;  /* zero input: SR result is draw-independent */
    uint8_t codes[AW4O_BLOCK];
    float s;
    aw4o_codec q = {cb, round_mode, zero_floor, eden, 1.0f, 1e-8f};
    quantize_block(&q, zeros, u, codes, &s);
    uint8_t byte = (uint8_t)(codes[0] | (codes[1] << 4));
    memset(packed, byte, (size_t)(n / 2));
    for (int64_t b = 0; b < n / AW4O_BLOCK; ++b) scales[b] = s;
    return 0;
}

int aw4o_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void aw4o_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
