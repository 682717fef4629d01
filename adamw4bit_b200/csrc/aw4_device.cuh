// aw4_device.cuh -- device helpers shared by the step and codec kernels.
//
// Numerics follow the reference's CPU semantics exactly (nubank/adamw4bit on
// PyTorch CPU): every float op below is an explicit IEEE round-to-nearest
// intrinsic so nvcc cannot contract or reassociate, and the library is also
// compiled with --fmad=false.  The only fused multiply-add is the one torch's
// lerp uses (m + w * (end - m) as one FMA, adamw.py:557, 684).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>
#include <type_traits>

#include "../../include/adamw4bit_b200.h"

namespace aw4 {

constexpr int kBlock = AW4_BLOCK;        // values per quantization block
constexpr int kPerLane = 8;              // consecutive values per thread
constexpr int kLanesPerBlock = kBlock / kPerLane;  // 16 threads per block
constexpr int kThreads = 256;            // threads per CTA
constexpr int kBlocksPerTile = kThreads / kLanesPerBlock;  // 16 blocks = 2048 values
constexpr float kScaleFloor = 1e-12f;    // quantization.py:706-712 (4-bit schemes)

// ---------------------------------------------------------------------------
// IEEE float32 ops (no contraction, no reassociation)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }
__device__ __forceinline__ float frcp(float a) { return __frcp_rn(a); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }

// torch.max / clamp propagate NaN; PTX max.NaN / min.NaN do the same.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ bool is_finite(float a) { return fabsf(a) < __int_as_float(0x7f800000); }

// Correctly rounded a / b from y = RN(1 / b) (Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990): q = RN(a*y) is within one ulp, the remainder
// r = a - q*b is exact in one FMA, and RN(q + r*y) is RN(a/b).  Preconditions
// (checked by the callers): b and y normal, and a == 0 or |a| >= 2^-100, so
// the quotient is normal and the remainder cannot underflow.
__device__ __forceinline__ float div_markstein(float a, float b, float y) {
    const float q = fmul(a, y);
    const float r = ffma(-q, b, a);
    return ffma(r, y, q);
}
constexpr float kMarksteinMinNumerator = 0x1p-100f;
constexpr float kMarksteinMaxDivisor = 0x1p26f;
constexpr float kMarksteinMinDivisor = 0x1p-100f;

// ---------------------------------------------------------------------------
// Reciprocal and square root from the hardware approximations, refined by
// one Newton-Raphson step (reciprocal) and one Markstein correction (square
// root): Markstein, IBM J. Res. Dev. 34(1), 1990; Muller et al., "Handbook of
// Floating-Point Arithmetic", 2nd ed., ch. 4-5.  Both are verified
// exhaustively against the IEEE round-to-nearest operations on the device
// (aw4_selfcheck_math, every float32 of their domains) before the kernels rely
// on them:
//   rcp_nr(b)  == RN(1/b)     for every b with 2^-126 <= |b| <= 2^126
//   sqrt_nr(x) == RN(sqrt(x)) for every x in [2^-102, 2^128) and x == 0
// (below 2^-102 the remainder x - s^2 underflows and sqrt_nr is not exact;
// the step only feeds it values scaled into range).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rcp_approx(float b) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    return y;
}
__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_nr(float b) {
    const float y = rcp_approx(b);
    const float e = ffma(-b, y, 1.0f);   // 1 - b*y, exact to one rounding
    return ffma(e, y, y);
}
constexpr float kNrMin = 0x1p-126f;
// x == 0 gives +0: the approximation reads max(x, 2^-126), so y is finite
// and every later product is a zero.
__device__ __forceinline__ float sqrt_nr(float x) {
    const float y = rsqrt_approx(fmaxf(x, kNrMin));
    const float s = fmul(x, y);
    const float h = fmul(0.5f, y);
    const float r = ffma(-s, s, x);      // x - s^2, exact
    return ffma(r, h, s);
}

// Three-input max/min (Blackwell).  max3_nan propagates NaN like torch.max;
// min3 ignores a NaN operand (its callers check finiteness separately).
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Max of |v[i]| over a lane's 8 values (NaN-propagating, like torch.max).
__device__ __forceinline__ float lane_absmax(const float v[8]) {
    float a = max3_nan(fabsf(v[0]), fabsf(v[1]), fabsf(v[2]));
    a = max3_nan(a, fabsf(v[3]), fabsf(v[4]));
    a = max3_nan(a, fabsf(v[5]), fabsf(v[6]));
    return max_nan(a, fabsf(v[7]));
}
// Min of |v[i]| over a lane's 8 values.
__device__ __forceinline__ float lane_absmin(const float v[8]) {
    float a = min3(fabsf(v[0]), fabsf(v[1]), fabsf(v[2]));
    a = min3(a, fabsf(v[3]), fabsf(v[4]));
    a = min3(a, fabsf(v[5]), fabsf(v[6]));
    return fminf(a, fabsf(v[7]));
}

// Min of a lane's 8 values (a NaN operand is ignored).
__device__ __forceinline__ float lane_min(const float v[8]) {
    float a = min3(v[0], v[1], v[2]);
    a = min3(a, v[3], v[4]);
    a = min3(a, v[5], v[6]);
    return fminf(a, v[7]);
}

// True if some value is a nonzero of magnitude below 2^-100 (such a lane
// takes the IEEE division path instead of div_markstein).  A lane whose
// smallest magnitude is at least 2^-100 is decided by one compare; otherwise
// (a zero, a tiny value or a NaN is present) the values are tested one by
// one: 2|v| - 1 in the integer domain maps zeros to the top of the range.
__device__ __forceinline__ bool any_tiny(const float v[8]) {
    if (lane_absmin(v) >= kMarksteinMinNumerator) return false;
    const uint32_t lim = 2u * (uint32_t)__float_as_int(kMarksteinMinNumerator) - 1u;
    uint32_t m = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = min(m, 2u * (uint32_t)__float_as_int(v[i]) - 1u);
    return m < lim;
}

// Branch-free form of any_tiny, for warp votes: the lane minimum decides
// most lanes; the exact per-value test is evaluated only when some lane of
// the warp needs it (the vote keeps that branch uniform).
__device__ __forceinline__ bool none_tiny_warp(const float v[8], bool lane_ok) {
    bool ok = lane_ok && lane_absmin(v) >= kMarksteinMinNumerator;
    if (!__all_sync(0xffffffffu, ok)) {
        const uint32_t lim = 2u * (uint32_t)__float_as_int(kMarksteinMinNumerator) - 1u;
        uint32_t m = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < 8; ++i) m = min(m, 2u * (uint32_t)__float_as_int(v[i]) - 1u);
        ok = lane_ok && m >= lim;
    }
    return ok;
}

// ---------------------------------------------------------------------------
// Packed float32 pairs (Blackwell f32x2, IEEE round-to-nearest).
// Only multiply and FMA are used.  ptxas may contract a packed multiply
// feeding a packed add/sub into one FMA (even with explicit .rn), so an
// addition is written as fma(a, one, b) with `one` a runtime 1.0 read from a
// kernel parameter: the product a*one is exact, the sum is rounded once, and
// no multiply can be fused into it.
// ---------------------------------------------------------------------------
typedef unsigned long long f2;
__device__ __forceinline__ f2 pk2(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk2(f2 r, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// d[i] = a[i] * b[i]
__device__ __forceinline__ void vmul8(float d[8], const float a[8], const float b[8]) {
#pragma unroll
    for (int i = 0; i < 8; i += 2)
        upk2(f2_mul(pk2(a[i], a[i + 1]), pk2(b[i], b[i + 1])), d[i], d[i + 1]);
}
// d[i] = a[i] * s
__device__ __forceinline__ void vmuls8(float d[8], const float a[8], float s) {
    const f2 ss = pk2(s, s);
#pragma unroll
    for (int i = 0; i < 8; i += 2) upk2(f2_mul(pk2(a[i], a[i + 1]), ss), d[i], d[i + 1]);
}
// d[i] = fma(s, a[i], c[i])
__device__ __forceinline__ void vfmas8(float d[8], float s, const float a[8], const float c[8]) {
    const f2 ss = pk2(s, s);
#pragma unroll
    for (int i = 0; i < 8; i += 2)
        upk2(f2_fma(ss, pk2(a[i], a[i + 1]), pk2(c[i], c[i + 1])), d[i], d[i + 1]);
}
// d[i] = RN(a[i] + b[i]), with one == 1.0 at run time
__device__ __forceinline__ void vadd8(float d[8], const float a[8], const float b[8], float one) {
    const f2 oo = pk2(one, one);
#pragma unroll
    for (int i = 0; i < 8; i += 2)
        upk2(f2_fma(pk2(a[i], a[i + 1]), oo, pk2(b[i], b[i + 1])), d[i], d[i + 1]);
}
// q[i] = RN(a[i] / b) with y = RN(1 / b) (div_markstein, pairwise)
__device__ __forceinline__ void vdiv_markstein8(float q[8], const float a[8], float b, float y) {
    const f2 bb = pk2(-b, -b), yy = pk2(y, y);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const f2 aa = pk2(a[i], a[i + 1]);
        const f2 q0 = f2_mul(aa, yy);
        const f2 r = f2_fma(q0, bb, aa);
        upk2(f2_fma(r, yy, q0), q[i], q[i + 1]);
    }
}

// ---------------------------------------------------------------------------
// Element IO: 8 consecutive values per thread, 16-byte vector accesses
// ---------------------------------------------------------------------------
template <int DT>
struct Elem;

template <>
struct Elem<AW4_F32> {
    static constexpr int kBytes = 4;
    __device__ __forceinline__ static void load8(const void* base, int64_t e, float v[8]) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + e);
        float4 a = __ldcs(p), b = __ldcs(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    __device__ __forceinline__ static void store8(void* base, int64_t e, const float v[8]) {
        float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + e);
        __stcs(p, make_float4(v[0], v[1], v[2], v[3]));
        __stcs(p + 1, make_float4(v[4], v[5], v[6], v[7]));
    }
    __device__ __forceinline__ static float round(float v) { return v; }
    __device__ __forceinline__ static float load1(const void* base, int64_t e) {
        return static_cast<const float*>(base)[e];
    }
    __device__ __forceinline__ static void store1(void* base, int64_t e, float v) {
        static_cast<float*>(base)[e] = v;
    }
};

// bf16: widening is exact; narrowing is round-to-nearest-even like c10::BFloat16.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct Elem<AW4_BF16> {
    static constexpr int kBytes = 2;
    __device__ __forceinline__ static void load8(const void* base, int64_t e, float v[8]) {
        uint4 w = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + e));
        v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x); v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
        v[4] = bf16_lo(w.z); v[5] = bf16_hi(w.z); v[6] = bf16_lo(w.w); v[7] = bf16_hi(w.w);
    }
    __device__ __forceinline__ static void store8(void* base, int64_t e, const float v[8]) {
        uint4 w = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                             pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        __stcs(reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + e), w);
    }
    __device__ __forceinline__ static float round(float v) {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
    __device__ __forceinline__ static float load1(const void* base, int64_t e) {
        return __uint_as_float(((uint32_t) static_cast<const uint16_t*>(base)[e]) << 16);
    }
    __device__ __forceinline__ static void store1(void* base, int64_t e, float v) {
        __nv_bfloat16 h = __float2bfloat16_rn(v);
        static_cast<uint16_t*>(base)[e] = *reinterpret_cast<uint16_t*>(&h);
    }
};

__device__ __forceinline__ float f16_lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float f16_hi(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    return (uint32_t)__half_as_ushort(__float2half_rn(lo)) |
           ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}

template <>
struct Elem<AW4_F16> {
    static constexpr int kBytes = 2;
    __device__ __forceinline__ static void load8(const void* base, int64_t e, float v[8]) {
        uint4 w = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + e));
        v[0] = f16_lo(w.x); v[1] = f16_hi(w.x); v[2] = f16_lo(w.y); v[3] = f16_hi(w.y);
        v[4] = f16_lo(w.z); v[5] = f16_hi(w.z); v[6] = f16_lo(w.w); v[7] = f16_hi(w.w);
    }
    __device__ __forceinline__ static void store8(void* base, int64_t e, const float v[8]) {
        uint4 w = make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]),
                             pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]));
        __stcs(reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + e), w);
    }
    __device__ __forceinline__ static float round(float v) {
        return __half2float(__float2half_rn(v));
    }
    __device__ __forceinline__ static float load1(const void* base, int64_t e) {
        return __half2float(__ushort_as_half(static_cast<const uint16_t*>(base)[e]));
    }
    __device__ __forceinline__ static void store1(void* base, int64_t e, float v) {
        static_cast<uint16_t*>(base)[e] = __half_as_ushort(__float2half_rn(v));
    }
};

// 8 consecutive gradient values summed over the ranks of an NVSwitch
// multicast object: `base` is the multicast address, and each 16-byte
// multimem.ld_reduce returns the element-wise sum of every rank's copy,
// reduced in the switch (BF16/F16 requested with FP32 accumulation and
// returned in the element type with the switch's own rounding, which on B200
// is not round-to-nearest-even; sums exact in the element type come back
// exactly).  Relaxed, system scope: the caller orders it after the
// ranks' writes with a cross-rank barrier.
template <int DT>
__device__ __forceinline__ void load8_reduce(const void* base, int64_t e, float v[8]);
template <>
__device__ __forceinline__ void load8_reduce<AW4_F32>(const void* base, int64_t e, float v[8]) {
    const float* p = static_cast<const float*>(base) + e;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]) : "l"(p) : "memory");
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]) : "l"(p + 4) : "memory");
}
template <>
__device__ __forceinline__ void load8_reduce<AW4_BF16>(const void* base, int64_t e, float v[8]) {
    const uint16_t* p = static_cast<const uint16_t*>(base) + e;
    uint32_t w[4];
    asm volatile(
        "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
        : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p) : "memory");
#pragma unroll
    for (int k = 0; k < 4; ++k) {   // element 2k in the low half
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void load8_reduce<AW4_F16>(const void* base, int64_t e, float v[8]) {
    const uint16_t* p = static_cast<const uint16_t*>(base) + e;
    uint32_t w[4];
    asm volatile(
        "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
        : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p) : "memory");
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[2 * k] = __half2float(__ushort_as_half((unsigned short)(w[k] & 0xffffu)));
        v[2 * k + 1] = __half2float(__ushort_as_half((unsigned short)(w[k] >> 16)));
    }
}

// The same reduction in two halves, so a caller can issue the next values'
// reduction before computing with the current ones: issue8_reduce starts the
// multimem.ld_reduce of 8 values into raw words (8 for FP32, 4 for 16-bit
// types), finish8_reduce widens them.  The loads are relaxed, system scope,
// ordered after the ranks' writes by the caller's cross-rank barrier.
template <int DT>
__device__ __forceinline__ void issue8_reduce(const void* base, int64_t e, uint32_t w[8]) {
    if constexpr (DT == AW4_F32) {
        const float* p = static_cast<const float*>(base) + e;
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p) : "memory");
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]) : "l"(p + 4) : "memory");
    } else if constexpr (DT == AW4_BF16) {
        const uint16_t* p = static_cast<const uint16_t*>(base) + e;
        asm volatile(
            "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
            : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p) : "memory");
    } else {
        const uint16_t* p = static_cast<const uint16_t*>(base) + e;
        asm volatile(
            "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
            : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p) : "memory");
    }
}
template <int DT>
__device__ __forceinline__ void finish8_reduce(const uint32_t w[8], float v[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if constexpr (DT == AW4_F32) {
            v[k] = __uint_as_float(w[k]);
        } else if constexpr (DT == AW4_BF16) {   // element 2j in the low half of word j
            v[k] = (k & 1) ? __uint_as_float(w[k >> 1] & 0xffff0000u)
                           : __uint_as_float(w[k >> 1] << 16);
        } else {
            v[k] = __half2float(__ushort_as_half(
                (unsigned short)((k & 1) ? (w[k >> 1] >> 16) : (w[k >> 1] & 0xffffu))));
        }
    }
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11).  Counter layout:
// (e/4 low word, e/4 high word, step, ordinal); key = 64-bit stream key;
// element e takes word e%4, top 24 bits -> uniform in [0, 1).
// ---------------------------------------------------------------------------
// The key schedule: round r uses (k0 + r*0x9E3779B9, k1 + r*0xBB67AE85).  The
// host computes it once per launch, so each round XORs kernel-parameter
// operands instead of advancing the key.
struct PhiloxKey {
    uint32_t k[20];   // (k0, k1) of rounds 0..9
};
inline PhiloxKey philox_schedule(uint64_t key) {
    PhiloxKey s;
    uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
    for (int r = 0; r < 10; ++r) {
        s.k[2 * r] = k0;
        s.k[2 * r + 1] = k1;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return s;
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, const PhiloxKey& K) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c.x;   // one widening multiply each
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.z;
        c = make_uint4((uint32_t)(p1 >> 32) ^ c.y ^ K.k[2 * r], (uint32_t)p1,
                       (uint32_t)(p0 >> 32) ^ c.w ^ K.k[2 * r + 1], (uint32_t)p0);
    }
    return c;
}

__device__ __forceinline__ float u24(uint32_t r) { return (float)(r >> 8) * 0x1p-24f; }
// The same draw scaled by 2^24: the integer r >> 8 as a float (exact).
__device__ __forceinline__ float k24(uint32_t r) { return (float)(r >> 8); }

// 8 uniforms for elements e .. e+7 (e a multiple of 4) of one stream; with
// SCALED, the uniforms times 2^24 (the preconditioner-space SR rule compares
// them with a probability scaled the same way).
template <bool SCALED = false>
__device__ __forceinline__ void philox_uniform8(const PhiloxKey& K, uint32_t step,
                                                uint32_t ordinal, uint64_t e, float u[8]) {
    const uint64_t q = e >> 2;
    uint4 r0 = philox4x32_10(make_uint4((uint32_t)q, (uint32_t)(q >> 32), step, ordinal), K);
    uint4 r1 = philox4x32_10(
        make_uint4((uint32_t)(q + 1), (uint32_t)((q + 1) >> 32), step, ordinal), K);
    const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) u[i] = SCALED ? k24(w[i]) : u24(w[i]);
}

// ---------------------------------------------------------------------------
// Rounding search (tables built by aw4_scheme_prepare)
// ---------------------------------------------------------------------------
// Rounding-search entry for bin edge b (x = -1 + 2b/N): the next threshold
// above the edge and the code at the edge.  For RTN schemes with the dyn4_nz
// floor the floor is folded in: codes below 1 read as 1.
struct __align__(8) SearchEntry {
    float next_thr;
    int code;
};
static_assert(sizeof(SearchEntry) == 8, "");

struct __align__(16) SmemScheme {
    SearchEntry tab[AW4_LUT_BINS + 1];   // the first lut_bins + 1 entries are used
    float cb[16];
    float half_bins;                      // lut_bins / 2
    float bias;                           // 2^23 + lut_bins / 2
};

__device__ __forceinline__ void load_scheme(SmemScheme& s, const aw4_scheme& g, int tid,
                                            int nthreads) {
    const bool floor_in_table = g.zero_floor && g.round_mode == AW4_RTN;
    const int nb = g.lut_bins;
    for (int b = tid; b <= nb; b += nthreads) {
        int k;
        if (b < nb) {
            k = g.lut[b];
        } else {  // edge x = 1.0: one more threshold may sit in the last bin
            k = g.lut[nb - 1];
            k += (g.thr[k + 1] <= 1.0f) ? 1 : 0;
        }
        float next = g.thr[k + 1];
        if (floor_in_table && k == 0) {
            // no threshold is at or below this bin's edge, so at most t1 lies
            // inside it, and max(code, 1) = 1 across the whole bin
            k = 1;
            next = INFINITY;
        }
        s.tab[b] = SearchEntry{next, k};
    }
    for (int i = tid; i < 16; i += nthreads) s.cb[i] = g.codebook[i];
    if (tid == 0) {
        s.half_bins = (float)(nb / 2);
        s.bias = 8388608.0f + (float)(nb / 2);
    }
}

// Per-lane register copies of a scheme's search constants and codebook level.
struct SchemeRegs {
    float cbv;             // cb[lane % 16], read by shuffles
    float half;            // lut_bins / 2
    float bias;            // 2^23 + lut_bins / 2
    uint32_t tab_biased;   // shared address of tab, minus 0x4B000000 * 8 (mod 2^32)
};
__device__ __forceinline__ SchemeRegs scheme_regs(const SmemScheme& s, int lane) {
    const uint32_t tab = static_cast<uint32_t>(__cvta_generic_to_shared(&s.tab[0]));
    return SchemeRegs{s.cb[lane & 15], s.half_bins, s.bias, tab - 0x4B000000u * 8u};
}

// Table search of a finite normalised value x in [-1, 1]: the stored code
// (RTN) or the searchsorted-left index (SR).  With N bins the edge index
// floor((x + 1) * N / 2) lands in the low mantissa bits of
// x * N/2 + (2^23 + N/2) when the FMA rounds toward zero (the power-of-two
// product is exact, the sum lies in [2^23, 2^23 + N] where float32 spacing is
// 1, and truncation of a positive value is its floor).
__device__ __forceinline__ int lut_search(const SmemScheme& s, const SchemeRegs& r, float x) {
    // entry address = bits * 8 + (table - 0x4B000000 * 8): the exponent bias
    // of the bin index folds into the table base (32-bit shared address)
    const uint32_t bits = __float_as_uint(__fmaf_rz(x, r.half, r.bias));
    const uint32_t addr = bits * 8u + r.tab_biased;
    float next;
    int count;
    asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=f"(next), "=r"(count) : "r"(addr));
    int ge;   // -1 if x >= next, else 0
    asm("set.ge.s32.f32 %0, %1, %2;" : "=r"(ge) : "f"(x), "f"(next));
    (void)s;
    return count - ge;
}

// lut_search of a pair of values, the bin indices computed by one packed
// round-toward-zero FMA.
__device__ __forceinline__ void lut_search2(const SchemeRegs& r, float x0, float x1, int code[2]) {
    f2 t;
    asm("fma.rz.f32x2 %0, %1, %2, %3;"
        : "=l"(t)
        : "l"(pk2(x0, x1)), "l"(pk2(r.half, r.half)), "l"(pk2(r.bias, r.bias)));
    float b0, b1;
    upk2(t, b0, b1);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t addr = __float_as_uint(k ? b1 : b0) * 8u + r.tab_biased;
        float next;
        int count, ge;
        asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=f"(next), "=r"(count) : "r"(addr));
        asm("set.ge.s32.f32 %0, %1, %2;" : "=r"(ge) : "f"(k ? x1 : x0), "f"(next));
        code[k] = count - ge;
    }
}

// lut_search over a lane's 8 values.
__device__ __forceinline__ void lut_search8(const SchemeRegs& r, const float x[8], int code[8]) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) lut_search2(r, x[i], x[i + 1], code + i);
}


// lut_search8 for an RTN scheme, returning the 8 codes packed as nibbles
// (value i in bits 4i..4i+3): code = count - ge (ge = -1 when x >= next) is
// accumulated as count * 16^i + ge * -16^i with integer multiply-adds.
__device__ __forceinline__ uint32_t lut_pack8(const SchemeRegs& r, const float x[8]) {
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        f2 t;
        asm("fma.rz.f32x2 %0, %1, %2, %3;" : "=l"(t)
            : "l"(pk2(x[i], x[i + 1])), "l"(pk2(r.half, r.half)), "l"(pk2(r.bias, r.bias)));
        float b0, b1;
        upk2(t, b0, b1);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t addr = __float_as_uint(k ? b1 : b0) * 8u + r.tab_biased;
            float next;
            int count, ge;
            asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=f"(next), "=r"(count) : "r"(addr));
            asm("set.ge.s32.f32 %0, %1, %2;" : "=r"(ge) : "f"(k ? x[i + 1] : x[i]), "f"(next));
            const uint32_t m = 1u << (4 * (i + k));
            asm("mad.lo.u32 %0, %1, %2, %0;" : "+r"(packed) : "r"(count), "r"(m));
            asm("mad.lo.u32 %0, %1, %2, %0;" : "+r"(packed) : "r"(ge), "r"(0u - m));
        }
    }
    return packed;
}

// Level of a code from the codebook held in registers: lane l keeps
// cbv = cb[l % 16], and a shuffle reads lane `code`.
__device__ __forceinline__ float level_of(float cbv, int code) {
    return __shfl_sync(0xffffffffu, cbv, code);
}

// Decodes 8 packed codes from the block's scaled codebook: lane 16h + k of
// the block's 16-lane group holds cbs = RN(cb[k] * scale), and a shuffle
// confined to the group reads lane `code` (the segment keeps only the low 4
// bits of the index, so w >> 4i needs no mask).  RN(cb[k] * scale) is the
// product decode8 forms.
__device__ __forceinline__ void decode8s(float cbs, uint32_t w, float v[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __shfl_sync(0xffffffffu, cbs, (int)(w >> (4 * i)), 16);
}

// torch.searchsorted(cb, x) (left): the ATen lower-bound loop, NaN -> 16.
__device__ __forceinline__ int searchsorted_left(const float* cb, float x) {
    int start = 0, end = 16;
    while (start < end) {
        const int mid = start + ((end - start) >> 1);
        if (!(cb[mid] >= x)) start = mid + 1; else end = mid;
    }
    return start;
}

// Literal RTN rule of quantization.py:263-272 (used for non-finite blocks).
__device__ __forceinline__ int rtn_literal(const float* cb, float x) {
    const int i = searchsorted_left(cb, x);
    const int l = max(i - 1, 0), r = min(i, 15);
    return (fabsf(fsub(x, cb[l])) < fabsf(fsub(cb[r], x))) ? l : r;
}

// Value-unbiased SR given the interval index (quantization.py:295-315).
__device__ __forceinline__ int value_sr_from_index(const float* cb, int i, float x, float u) {
    const int l = max(i - 1, 0), r = min(i, 15);
    const float a = cb[l], b = cb[r];
    const float width = fsub(b, a);
    float p = fdiv(fsub(x, a), max_nan(width, 1e-12f));
    p = (width > 0.0f) ? p : 0.0f;
    p = min_nan(max_nan(p, 0.0f), 1.0f);
    return (u < p) ? r : l;
}

// Adam preconditioner 1 / (sqrt(max(s * l / bias, 0)) + eps) (quantization.py:356-358).
__device__ __forceinline__ float precond(float s, float level, float bias, float eps) {
    return frcp(fadd(fsqrt(max_nan(fdiv(fmul(s, level), bias), 0.0f)), eps));
}

// Preconditioner-space SR given the interval index and the block's level
// preconditioners f[k] = precond(s, cb[k]) (quantization.py:336-377).
__device__ __forceinline__ int update_sr_from_index(const float* cb, const float* f, int i,
                                                    float x, float s, float bias, float eps,
                                                    float u) {
    const int l = max(i - 1, 0), r = min(i, 15);
    const float width = fsub(cb[r], cb[l]);
    const float fl = f[l], fr = f[r];
    const float fx = precond(s, x, bias, eps);
    const float den = fsub(fl, fr);
    float p = fdiv(fsub(fx, fr), max_nan(den, 1e-30f));
    p = (width > 0.0f && den > 0.0f) ? p : 1.0f;
    p = min_nan(max_nan(p, 0.0f), 1.0f);
    return (u < p) ? l : r;
}

// Max over the 16 lanes of a block group (lanes 16h .. 16h+15 of a warp),
// NaN-propagating like torch.max: two full-warp reductions (Blackwell
// redux.f32), one per group, to which the other group's lanes contribute
// -inf.  The whole warp must call it.  One reduction per group with a
// half-warp member mask gives the same values, but the two masks within one
// warp cost convergence handling that made the step kernel 5 % slower.
__device__ __forceinline__ float group_max16(float v) {
    const bool hi = (threadIdx.x & 16) != 0;
    const float lo_in = hi ? -INFINITY : v, hi_in = hi ? v : -INFINITY;
    float r0, r1;
    asm volatile("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r0) : "f"(lo_in));
    asm volatile("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r1) : "f"(hi_in));
    return hi ? r1 : r0;
}

}  // namespace aw4
