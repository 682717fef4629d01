// aw4_encode.cuh -- block encoder shared by the fused step and the codec.
//
// A 128-value block is held by a group of 16 consecutive lanes, 8 values
// each (lane j holds values 8j .. 8j+7).  The encoder reproduces
// quantization.py:_quantize_impl (lines 937-960) for 4-bit codebooks:
//   scale = max(absmax(block), 1e-12); x = v / scale; codes by RTN or SR;
//   optional zero floor (dyn4_nz); optional EDEN scale calibration.
#pragma once

#include "aw4_device.cuh"

namespace aw4 {

// Per-warp scratch for EDEN sums and the update-SR level table.
// EDEN: four tables (num/den x the warp's 2 groups) of 16 rows x 12 floats
// (8 products + 4 pad).  The 12-float rows make each quarter-warp's float4
// row writes hit 32 distinct banks; tables 200 floats apart start 8 banks
// apart, so the 32 lanes' column reads hit 32 distinct banks too.
constexpr int kEdenRow = 12;
constexpr int kEdenTable = 200;
constexpr int kWarpScratch = 4 * kEdenTable + 32 /* update-SR level tables */;

struct GroupCtx {
    float* eden_num;   // this group's products tables
    float* eden_den;
    float* levels;     // 16 floats: update-SR preconditioner of each level
    int j;             // lane within the group (0..15)
    int lane;          // lane within the warp
};

__device__ __forceinline__ GroupCtx group_ctx(float* warp_scratch, int lane) {
    const int h = lane >> 4;
    GroupCtx g;
    g.eden_num = warp_scratch + (2 * h) * kEdenTable;
    g.eden_den = warp_scratch + (2 * h + 1) * kEdenTable;
    g.levels = warp_scratch + 4 * kEdenTable + 16 * h;
    g.j = lane & 15;
    g.lane = lane;
    return g;
}

// Sum of the block's 128 products in torch's CPU reduction order for
// (nb, 128).sum(dim=1): vector v (values 8v .. 8v+7) accumulates into
// accumulator v % 4, the accumulators combine in order, then the 8 lanes are
// summed in order from zero.  Lane j of the group holds vector v = j.
// Returns (num, den) totals, valid in every lane of the group.
__device__ __forceinline__ float2 eden_sums(const GroupCtx& g, const float np[8],
                                            const float dp[8]) {
    float4* rn = reinterpret_cast<float4*>(g.eden_num + kEdenRow * g.j);
    float4* rd = reinterpret_cast<float4*>(g.eden_den + kEdenRow * g.j);
    rn[0] = make_float4(np[0], np[1], np[2], np[3]);
    rn[1] = make_float4(np[4], np[5], np[6], np[7]);
    rd[0] = make_float4(dp[0], dp[1], dp[2], dp[3]);
    rd[1] = make_float4(dp[4], dp[5], dp[6], dp[7]);
    __syncwarp();
    // lanes 0-7: numerator column c; lanes 8-15: denominator column c
    const float* tab = (g.j < 8) ? g.eden_num : g.eden_den;
    const int c = g.j & 7;
    float acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float a = fadd(0.0f, tab[kEdenRow * k + c]);
        a = fadd(a, tab[kEdenRow * (k + 4) + c]);
        a = fadd(a, tab[kEdenRow * (k + 8) + c]);
        a = fadd(a, tab[kEdenRow * (k + 12) + c]);
        acc[k] = a;
    }
    const float t = fadd(fadd(fadd(acc[0], acc[1]), acc[2]), acc[3]);
    __syncwarp();  // tables are reused by the next block
    // column totals in order from zero: each lane chains its half's 8 totals
    const int base = g.lane & 24;   // group base + numerator/denominator half
    float chain = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) chain = fadd(chain, __shfl_sync(0xffffffffu, t, base + i));
    const float num = __shfl_sync(0xffffffffu, chain, g.lane & 16);
    const float den = __shfl_sync(0xffffffffu, chain, (g.lane & 16) | 8);
    return make_float2(num, den);
}

// Max of |v[i]| over a lane's 8 values (NaN-propagating, like torch.max).
__device__ __forceinline__ float lane_absmax(const float v[8]) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a = max_nan(a, fabsf(v[i]));
    return a;
}

// Encodes the group's block.  v: this lane's 8 working values; amax: their
// lane_absmax.  u: 8 uniforms (SR modes).  Returns this lane's 8 codes packed
// as nibbles (value 8j+i in bits 4i..4i+3, i.e. the reference's little-endian
// nibble order) and sets *scale_out to the block scale to store (identical
// in all 16 lanes).
template <int MODE>
__device__ __forceinline__ uint32_t encode_block(const SmemScheme& S, const SchemeRegs& R,
                                                 const GroupCtx& g,
                                                 const float v[8], float amax, const float u[8],
                                                 int zero_floor, int eden, float sr_bias,
                                                 float sr_eps, float* scale_out) {
    amax = group_max16(amax);
    const float sc = max_nan(amax, kScaleFloor);
    const bool fin = is_finite(sc);
    if (MODE == AW4_SR_UPDATE) {
        g.levels[g.j] = precond(sc, S.cb[g.j], sr_bias, sr_eps);
        __syncwarp();
    }
    // x = v / scale, correctly rounded (Markstein when its preconditions
    // hold).  A nonzero |v| < 2^-100 gives |x| < 2^-99, which every supported
    // codebook rounds (RTN) to the code of 0 whatever its last bits, so RTN
    // without EDEN needs no guard for it.
    float x[8], q[8];
    int code[8];
    if (fin) {
        const bool need_guard = (MODE != AW4_RTN) || eden;
        if (sc <= kMarksteinMaxDivisor && !(need_guard && any_tiny(v))) {
            vdiv_markstein8(x, v, sc, frcp(sc));
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = fdiv(v[i], sc);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = lut_search(S, R, x[i]);
            if (MODE == AW4_RTN) {
                code[i] = idx;  // the dyn4_nz floor is folded into the RTN table
            } else {
                code[i] = (MODE == AW4_SR_VALUE)
                              ? value_sr_from_index(S.cb, idx, x[i], u[i])
                              : update_sr_from_index(S.cb, g.levels, idx, x[i], sc, sr_bias,
                                                     sr_eps, u[i]);
                if (zero_floor) code[i] = max(code[i], 1);
            }
        }
    } else {
        // non-finite block (NaN/inf moments): the literal reference rules
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x[i] = fdiv(v[i], sc);
            if (MODE == AW4_RTN) {
                code[i] = rtn_literal(S.cb, x[i]);
            } else {
                const int idx = searchsorted_left(S.cb, x[i]);
                code[i] = (MODE == AW4_SR_VALUE)
                              ? value_sr_from_index(S.cb, idx, x[i], u[i])
                              : update_sr_from_index(S.cb, g.levels, idx, x[i], sc, sr_bias,
                                                     sr_eps, u[i]);
            }
            if (zero_floor) code[i] = max(code[i], 1);
        }
    }
    if (MODE == AW4_SR_UPDATE) __syncwarp();  // level table reused by the next block
    float s = sc;
    if (eden) {
        float np[8], dp[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = level_of(R.cbv, code[i]);
        vmul8(np, x, x);
        vmul8(dp, x, q);
        const float2 nd = eden_sums(g, np, dp);
        s = fmul(sc, fdiv(nd.x, max_nan(nd.y, kScaleFloor)));
    }
    *scale_out = s;
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) packed |= (uint32_t)code[i] << (4 * i);
    return packed;
}

}  // namespace aw4
