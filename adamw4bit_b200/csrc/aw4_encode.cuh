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

// Per-warp scratch for EDEN sums and the update-SR level tables.
//
// EDEN products go to four column-major tables per warp (numerator and
// denominator for each of the warp's two groups): 8 columns of 16 rows, with
// a column stride of 20 floats.  A lane (row j) writes its 8 products to
// address 20c + j: the two groups' tables start 16 banks apart, so the 32
// lanes of each store hit 32 distinct banks.  A reading lane takes one whole
// column as four float4 (rows 4k .. 4k+3); with the 20-float stride the 8
// columns of a quarter-warp start in 8 distinct 4-bank groups.  Column totals
// are then exchanged through 16 floats per group, interleaved as
// (numerator, denominator) pairs.
constexpr int kEdenCol = 20;                       // column stride (16 rows + 4 pad)
constexpr int kEdenTable = 8 * kEdenCol;           // 160 floats
// group h: numerator table at 336h, denominator table at 160 + 336h
constexpr int kEdenDen = 160;                      // denominator table offset
constexpr int kEdenGroup = 336;                    // second group's offset (16 mod 32)
constexpr int kEdenTotals = 656;                   // 2 groups x 16 floats
constexpr int kSrLevels = kEdenTotals + 32;        // 2 groups x 16 floats
constexpr int kSrTable = kSrLevels + 32;           // 2 groups x 17 float4
constexpr int kWarpScratch = kSrTable + 136;       // 856 floats
static_assert(kSrTable % 4 == 0, "float4 table");

// RN(1 / bias) for the fast update-SR encoder, or 0 (fast encoder off) unless
// bias lies in [2^-40, 1] and eps in [2^-60, 2^25], the ranges its exactness
// argument covers (codebooks lie in [-1, 1], checked by aw4_scheme_prepare).
// Host code: the float32 division is correctly rounded.
inline float sr_fast_rbias(float bias, float eps) {
    if (!(bias >= 0x1p-40f && bias <= 1.0f && eps >= 0x1p-60f && eps <= 0x1p25f)) return 0.0f;
    volatile float one = 1.0f;
    return one / bias;
}
static_assert(kEdenGroup % 32 == 16 && kEdenDen % 32 == 0, "bank offsets");
static_assert(kEdenDen >= kEdenTable && kEdenGroup >= kEdenDen + kEdenTable, "tables overlap");
static_assert(kEdenTotals >= kEdenGroup + kEdenDen + kEdenTable && kEdenTotals % 4 == 0, "");

struct GroupCtx {
    float* tab_num;    // this group's column-major product tables
    float* tab_den;
    const float* rd;   // the column this lane reduces (numerator or denominator table)
    float* totals;     // this group's 16 interleaved column totals
    float* levels;     // 16 floats: update-SR preconditioner of each level
    float4* sr_tab;    // 17 entries: the fast update-SR rule's interval table
    int j;             // lane within the group (0..15)
    int lane;          // lane within the warp
    float one;         // 1.0 at run time (packed additions)
};

__device__ __forceinline__ GroupCtx group_ctx(float* warp_scratch, int lane, float one) {
    const int h = lane >> 4;
    GroupCtx g;
    g.tab_num = warp_scratch + kEdenGroup * h;
    g.tab_den = warp_scratch + kEdenDen + kEdenGroup * h;
    g.j = lane & 15;
    g.rd = (g.j < 8 ? g.tab_num : g.tab_den) + kEdenCol * (g.j & 7);
    g.totals = warp_scratch + kEdenTotals + 16 * h;
    g.levels = warp_scratch + kSrLevels + 16 * h;
    g.sr_tab = reinterpret_cast<float4*>(warp_scratch + kSrTable) + 17 * h;
    g.lane = lane;
    g.one = one;
    return g;
}

// Sums of the block's 128 numerator and denominator products in torch's CPU
// reduction order for (nb, 128).sum(dim=1): vector v (values 8v .. 8v+7)
// accumulates into accumulator v % 4, the four accumulators combine in
// order, then the 8 vector lanes are summed in order.  Lane j of the group
// holds vector v = j.  The leading "0 +" of each chain is dropped: it can
// only turn a -0 into +0, and the sums feed max(den, 1e-12) and a quotient
// whose numerator is a sum of squares, so zero signs never reach a result.
// Returns (num, den), valid in every lane of the group.
// eden_write stores a lane's products; eden_finish (after independent work,
// if any) reduces them.
__device__ __forceinline__ void eden_write(const GroupCtx& g, const float np[8],
                                           const float dp[8]) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        g.tab_num[kEdenCol * c + g.j] = np[c];
        g.tab_den[kEdenCol * c + g.j] = dp[c];
    }
}
__device__ __forceinline__ float2 eden_finish(const GroupCtx& g) {
    __syncwarp();
    // lanes 0-7: numerator column j; lanes 8-15: denominator column j - 8
    const float4* col = reinterpret_cast<const float4*>(g.rd);
    const float4 r0 = col[0], r1 = col[1], r2 = col[2], r3 = col[3];
    const f2 oo = pk2(g.one, g.one);
    // (acc0, acc1) over rows (0,1), (4,5), (8,9), (12,13); (acc2, acc3) likewise
    f2 a01 = pk2(r0.x, r0.y), a23 = pk2(r0.z, r0.w);
    a01 = f2_fma(pk2(r1.x, r1.y), oo, a01);
    a23 = f2_fma(pk2(r1.z, r1.w), oo, a23);
    a01 = f2_fma(pk2(r2.x, r2.y), oo, a01);
    a23 = f2_fma(pk2(r2.z, r2.w), oo, a23);
    a01 = f2_fma(pk2(r3.x, r3.y), oo, a01);
    a23 = f2_fma(pk2(r3.z, r3.w), oo, a23);
    float acc0, acc1, acc2, acc3;
    upk2(a01, acc0, acc1);
    upk2(a23, acc2, acc3);
    const float t = fadd(fadd(fadd(acc0, acc1), acc2), acc3);
    g.totals[2 * (g.j & 7) + (g.j >> 3)] = t;
    __syncwarp();
    const float4* tot = reinterpret_cast<const float4*>(g.totals);
    const float4 t0 = tot[0], t1 = tot[1], t2 = tot[2], t3 = tot[3];
    // (num, den) chained over the 8 columns in order
    f2 ch = pk2(t0.x, t0.y);
    ch = f2_fma(pk2(t0.z, t0.w), oo, ch);
    ch = f2_fma(pk2(t1.x, t1.y), oo, ch);
    ch = f2_fma(pk2(t1.z, t1.w), oo, ch);
    ch = f2_fma(pk2(t2.x, t2.y), oo, ch);
    ch = f2_fma(pk2(t2.z, t2.w), oo, ch);
    ch = f2_fma(pk2(t3.x, t3.y), oo, ch);
    ch = f2_fma(pk2(t3.z, t3.w), oo, ch);
    __syncwarp();  // tables and totals are reused by the next block
    float num, den;
    upk2(ch, num, den);
    return make_float2(num, den);
}
__device__ __forceinline__ float2 eden_sums(const GroupCtx& g, const float np[8],
                                            const float dp[8]) {
    eden_write(g, np, dp);
    return eden_finish(g);
}

// 2^24 precond(s, level): the fast exact sequence (Markstein by the bias,
// sqrt_nr, rcp_nr of the scaled sum) when s*level is 0 or at least 2^-100
// (so s*level/bias is 0 or in sqrt_nr's exact range), else the IEEE
// operations.  Scaling the last sum by 2^-24 is exact (it stays normal), so
// the reciprocal is 2^24 RN(1/(root + eps)).
__device__ __forceinline__ float precond24(float s, float level, float bias, float rbias,
                                           float eps) {
    const float t = fmul(s, level);
    if (t == 0.0f || t >= kMarksteinMinNumerator) {
        const float root = sqrt_nr(div_markstein(t, bias, rbias));
        return rcp_nr(ffma(root, 0x1p-24f, fmul(eps, 0x1p-24f)));
    }
    return fmul(precond(s, level, bias, eps), 0x1p24f);
}

// The fast update-SR rule's per-block table (quantization.py:336-377 with the
// reference's f[k] = precond(s, cb[k])).  Entry i, for the searchsorted-left
// index i of a value (l = max(i-1, 0), r = min(i, 15)):
//   x: 2^24 f[r]
//   y: the quotient's divisor f[l] - f[r]
//   z: RN(1 / divisor), or 0 where the code does not depend on the draw
//   w: the code taken when the draw is not below p (int bits)
// With the zero floor applied to both codes, entries whose two codes
// coincide, and intervals for which the reference sets p = 1 (no positive
// width or divisor: the code is l for every draw in [0, 1)), have z = 0, so
// the Markstein quotient is zero and code w is taken.  Preconditions (host
// and caller): bias in [2^-40, 1], eps in [2^-60, 2^25], s <= 2^26 and
// |cb| <= 1.  Then every f lies in [2^-34, 2^60], so a positive divisor lies
// in [2^-57, 2^60], inside rcp_nr's exact range.
__device__ __forceinline__ void sr_table(const GroupCtx& g, const SmemScheme& S, float sc,
                                         int floor_code, float bias, float rbias, float eps) {
    const int j = g.j;
    const float fj = precond24(sc, S.cb[j], bias, rbias, eps);
    const float fprev = __shfl_up_sync(0xffffffffu, fj, 1, 16);
    // branch-free: lane 0 has no interval below it (its fprev is its own fj)
    const int rc0 = max(j, floor_code), lc = max(j - 1, floor_code);
    const float den = fsub(fprev, fj);   // 2^24 (f[l] - f[r]), exactly
    const bool interval = j >= 1 && fsub(S.cb[j], S.cb[max(j - 1, 0)]) > 0.0f && den > 0.0f;
    const float dl = interval ? fmul(den, 0x1p-24f) : 1.0f;
    const float yr = rcp_nr(dl);        // dl is 1 or a normal divisor in rcp_nr's exact range
    const float y = (interval && lc != rc0) ? yr : 0.0f;
    const int rc = (j >= 1 && !interval) ? lc : rc0;
    g.sr_tab[j] = make_float4(fj, dl, y, __int_as_float(rc));
    if (j == 15) g.sr_tab[16] = make_float4(fj, 1.0f, 0.0f, __int_as_float(15));
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
            vdiv_markstein8(x, v, sc, rcp_nr(sc));
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
                                                     sr_eps, fmul(u[i], 0x1p-24f));
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
                                                     sr_eps, fmul(u[i], 0x1p-24f));
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
        // s' = s * (sum x^2 / max(sum x*q, 1e-12)); the divisor lies in
        // [1e-12, 128] (|x| <= 1, |q| <= 1), so Markstein applies unless the
        // numerator is a nonzero below 2^-100 or a sum is not finite (NaN
        // fails every compare)
        const float dd = max_nan(nd.y, kScaleFloor);
        const float ratio = (dd <= kMarksteinMaxDivisor &&
                             (nd.x == 0.0f ||
                              (nd.x >= kMarksteinMinNumerator && nd.x <= 0x1p100f)))
                                ? div_markstein(nd.x, dd, rcp_nr(dd))
                                : fdiv(nd.x, dd);
        s = fmul(sc, ratio);
    }
    *scale_out = s;
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) packed += (uint32_t)code[i] << (4 * i);   // disjoint nibbles
    return packed;
}

// The fast update-SR rule over a lane's 8 values, pair by pair: x = v/s by
// Markstein, the searchsorted index, 2^24 fx by the fast sequence of
// precond24 (packed where no operand needs a sign change), the table entry of
// the index, the quotient p' = 2^24 (fx - f[r]) / (f[l] - f[r]) by Markstein,
// and code = w - (u' < p') with u' = 2^24 u.  Ranges, beyond the table's: v
// is non-negative (an m2 moment, or the codec's vote) and 0 or >= 2^-100, so
// s*x is 0 or >= 2^-101, s*x/bias is 0 or in [2^-101, 2^66] and exact by
// Markstein, and root + eps lies in [2^-60, 2^34]; 2^24 fx and 2^24 f[r] lie
// in [2^-10, 2^84], so a nonzero difference is at least 2^-33, and the
// quotient, in [0, 2^24] because precond is non-increasing and x lies in
// [cb[l], cb[r]], is normal with an exact remainder.  The reference's clamp
// of p to [0, 1] is then the identity.  Returns the packed codes.
__device__ __forceinline__ uint32_t encode_fast_upd_sr(const SchemeRegs& R, const GroupCtx& g,
                                                       const float v[8], float sc,
                                                       const float u[8], float bias,
                                                       float rbias, float eps) {
    const float ys = rcp_nr(sc);
    const f2 nsc = pk2(-sc, -sc), yss = pk2(ys, ys), scp = pk2(sc, sc);
    const f2 rb = pk2(rbias, rbias), nb = pk2(-bias, -bias);
    const f2 hh = pk2(0.5f, 0.5f);
    const float eps24 = fmul(eps, 0x1p-24f);
    const f2 nee = pk2(-eps24, -eps24), ns24 = pk2(-0x1p-24f, -0x1p-24f);
    const f2 one2 = pk2(g.one, g.one), tiny = pk2(kNrMin, kNrMin);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        // x = v / s (Markstein)
        const f2 vv = pk2(v[i], v[i + 1]);
        const f2 xq = f2_mul(vv, yss);
        const f2 xx = f2_fma(f2_fma(xq, nsc, vv), yss, xq);
        float x0, x1;
        upk2(xx, x0, x1);
        int idx[2];
        lut_search2(R, x0, x1, idx);
        // s*x / bias (Markstein)
        const f2 t1 = f2_mul(xx, scp);
        const f2 q0 = f2_mul(t1, rb);
        const f2 t2 = f2_fma(f2_fma(q0, nb, t1), rb, q0);
        float ta, tb;
        upk2(t2, ta, tb);
        // sqrt_nr of both; the approximation reads t + 2^-126, which is t
        // for every nonzero t (>= 2^-101) and 2^-126 for t == 0
        float ga, gb;
        upk2(f2_fma(t2, one2, tiny), ga, gb);
        const f2 y = pk2(rsqrt_approx(ga), rsqrt_approx(gb));
        const f2 sq = f2_mul(t2, y), h = f2_mul(hh, y);
        float sa, sb;
        upk2(sq, sa, sb);
        const f2 root = f2_fma(pk2(ffma(-sa, sa, ta), ffma(-sb, sb, tb)), h, sq);
        // rcp_nr of d = 2^-24 (root + eps), both, from nd = -d
        const f2 nd = f2_fma(root, ns24, nee);
        float na, nb;
        upk2(nd, na, nb);
        const float ra = rcp_approx(-na), rbb = rcp_approx(-nb);
        const f2 yy = pk2(ra, rbb);
        float fa, fb;
        upk2(f2_fma(f2_fma(nd, yy, one2), yy, yy), fa, fb);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float4 t = g.sr_tab[idx[k]];
            const float pq = div_markstein(fsub(k ? fb : fa, t.x), t.y, t.z);
            const int code = __float_as_int(t.w) - (u[i + k] < pq ? 1 : 0);
            packed += (uint32_t)code << (4 * (i + k));   // disjoint nibbles
        }
    }
    return packed;
}

// encode_block for a warp whose blocks all meet the fast preconditions (the
// caller has voted): a finite scale sc = max(absmax, 1e-12) <= 2^26; for SR
// or EDEN, no nonzero value below 2^-100; for EDEN, absmax >= 1e-12.  The same results as
// encode_block, without its per-lane branches.  It runs in two parts so a
// caller can put independent work between them: encode_fast_codes returns the
// packed codes and, with EDEN, leaves the products in the group's tables;
// encode_fast_scale then returns the block scale to store.
template <int MODE>
__device__ __forceinline__ uint32_t encode_fast_codes(const SmemScheme& S, const SchemeRegs& R,
                                                      const GroupCtx& g, const float v[8],
                                                      float sc, const float u[8], int zero_floor,
                                                      int eden, float sr_bias, float sr_eps,
                                                      float sr_rbias, float one) {
    const int floor_code = (MODE != AW4_RTN && zero_floor) ? 1 : 0;
    if (MODE == AW4_SR_UPDATE && sr_rbias > 0.0f && !eden) {   // launch-uniform
        sr_table(g, S, sc, floor_code, sr_bias, sr_rbias, sr_eps);
        __syncwarp();
        const uint32_t packed = encode_fast_upd_sr(R, g, v, sc, u, sr_bias, sr_rbias, sr_eps);
        __syncwarp();   // the table is rebuilt for the next block
        return packed;
    }
    if (MODE == AW4_SR_UPDATE) {
        g.levels[g.j] = precond(sc, S.cb[g.j], sr_bias, sr_eps);
        __syncwarp();
    }
    float x[8];
    int code[8];
    vdiv_markstein8(x, v, sc, rcp_nr(sc));
    if (MODE == AW4_RTN && !eden) return lut_pack8(R, x);
    int idxs[8];
    lut_search8(R, x, idxs);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int idx = idxs[i];
        if (MODE == AW4_RTN) {
            code[i] = idx;  // the dyn4_nz floor is folded into the RTN table
        } else {
            code[i] = (MODE == AW4_SR_VALUE)
                          ? value_sr_from_index(S.cb, idx, x[i], u[i])
                          : update_sr_from_index(S.cb, g.levels, idx, x[i], sc, sr_bias, sr_eps,
                                                 fmul(u[i], 0x1p-24f));
            code[i] = max(code[i], floor_code);
        }
    }
    if (MODE == AW4_SR_UPDATE) __syncwarp();  // level table reused by the next block
    if (eden) {
        float q[8], np[8], dp[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = level_of(R.cbv, code[i]);
        vmul8(np, x, x);
        vmul8(dp, x, q);
        eden_write(g, np, dp);
    }
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) packed += (uint32_t)code[i] << (4 * i);   // disjoint nibbles
    return packed;
}

// With EDEN the fast path also requires absmax >= 1e-12, so sc is the block's
// absmax and its largest element normalises to exactly +-1, a codebook level
// of every supported scheme (coded to itself by RTN and by both SR rules).
// Both sums then hold a term equal to 1 among non-negative terms: they lie in
// [1, 128], max(den, 1e-12) is den, and Markstein's preconditions hold.
__device__ __forceinline__ float encode_fast_scale(const GroupCtx& g, float sc, int eden) {
    if (!eden) return sc;
    const float2 nd = eden_finish(g);
    return fmul(sc, div_markstein(nd.x, nd.y, rcp_nr(nd.y)));
}

template <int MODE>
__device__ __forceinline__ uint32_t encode_fast(const SmemScheme& S, const SchemeRegs& R,
                                                const GroupCtx& g, const float v[8], float sc,
                                                const float u[8], int zero_floor, int eden,
                                                float sr_bias, float sr_eps, float sr_rbias,
                                                float one, float* scale_out) {
    const uint32_t c = encode_fast_codes<MODE>(S, R, g, v, sc, u, zero_floor, eden, sr_bias,
                                               sr_eps, sr_rbias, one);
    *scale_out = encode_fast_scale(g, sc, eden);
    return c;
}

}  // namespace aw4
