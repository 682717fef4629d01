// aw4_host.cu -- ABI identity, error reporting and aw4_scheme_prepare.
//
// aw4_scheme_prepare turns one of the reference's sorted 16-level codebooks
// (quantization.py:401-552) into the tables the kernels round with.  RTN's
// rule -- searchsorted-left, then the nearer neighbour with ties to the upper
// level (quantization.py:263-272) -- is a monotone step function of the
// normalised value, so it is fully described by 15 float32 thresholds
// t_k = min{x : code(x) >= k}, found here by bisection over the ordered
// float32 line with the literal rule.  For SR the search needs the
// searchsorted index itself, i = #{k : cb[k] < x} = #{k : x >= nextup(cb[k])}.
// A table of N uniform bins over [-1, 1] (N the fewest power of two, at most
// 1024, for which no bin holds two thresholds) then gives each bin's count of
// thresholds at its lower edge.  The kernels compute the bin exactly,
// floor((x + 1) * N / 2), with a round-toward-zero FMA (the power-of-two
// product is exact and rounding toward zero never crosses an integer), so
// one compare against the next threshold finishes the search.  The tables
// are verified against the literal rule before they are returned.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/adamw4bit_b200.h"
#include "aw4_host.h"

namespace aw4 {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

int32_t fail(int32_t code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static uint32_t fbits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
static float bitsf(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
// Monotone map of non-NaN floats to integers (+0 and -0 both map to 0).
static int64_t fkey(float f) {
    const uint32_t u = fbits(f);
    return (u & 0x80000000u) ? -(int64_t)(u & 0x7fffffffu) : (int64_t)u;
}
static float keyf(int64_t k) {
    return k < 0 ? bitsf(0x80000000u | (uint32_t)(-k)) : bitsf((uint32_t)k);
}

// quantization.py:263-272, evaluated in float32 on the host.
static int searchsorted_left(const float* cb, float x) {
    int start = 0, end = 16;
    while (start < end) {
        int mid = start + ((end - start) >> 1);
        if (!(cb[mid] >= x)) start = mid + 1; else end = mid;
    }
    return start;
}
static int rtn_literal(const float* cb, float x) {
    const int i = searchsorted_left(cb, x);
    const int l = i - 1 < 0 ? 0 : i - 1, r = i > 15 ? 15 : i;
    volatile float dl = std::fabs(x - cb[l]);
    volatile float dr = std::fabs(cb[r] - x);
    return dl < dr ? l : r;
}

// Host copy of the kernels' table search (x in [-1, 1]); the edge at x == 1
// extends the last bin's count by the threshold it may hold.
static int lut_search(const aw4_scheme& s, float x) {
    const int half = s.lut_bins / 2;
    volatile float t = x * (float)half;   // exact (power-of-two scale)
    const int b = (int)std::floor(t) + half;
    int k;
    if (b < s.lut_bins) {
        k = s.lut[b];
    } else {
        k = s.lut[s.lut_bins - 1];
        k += (s.thr[k + 1] <= 1.0f) ? 1 : 0;
    }
    return k + (x >= s.thr[k + 1] ? 1 : 0);
}

static int expected(const aw4_scheme& s, float x) {
    return s.round_mode == AW4_RTN ? rtn_literal(s.codebook, x) : searchsorted_left(s.codebook, x);
}

}  // namespace aw4

using namespace aw4;

extern "C" int32_t aw4_abi_version(void) { return AW4_ABI_VERSION; }

extern "C" const char* aw4_last_error(void) { return g_last_error.c_str(); }

extern "C" uint64_t aw4_launch_count(void) { return g_launches.load(); }

extern "C" int32_t aw4_scheme_prepare(const float* cb, int32_t round_mode, int32_t zero_floor,
                                      aw4_scheme* out) {
    if (!cb || !out) return fail(AW4_ERR_INVALID, "aw4_scheme_prepare: null argument");
    if (round_mode < AW4_RTN || round_mode > AW4_SR_UPDATE)
        return fail(AW4_ERR_INVALID, "aw4_scheme_prepare: bad round mode %d", round_mode);
    for (int k = 0; k < 16; ++k) {
        if (!std::isfinite(cb[k]) || cb[k] < -1.0f || cb[k] > 1.0f)
            return fail(AW4_ERR_UNSUPPORTED, "codebook level %d outside [-1, 1]", k);
        if (k && !(cb[k] > cb[k - 1]))
            return fail(AW4_ERR_INVALID, "codebook is not strictly increasing at %d", k);
    }
    if (cb[15] != 1.0f)
        return fail(AW4_ERR_UNSUPPORTED, "codebook must end at 1.0 (absmax scaling)");
    aw4_scheme s;
    std::memset(&s, 0, sizeof(s));
    std::memcpy(s.codebook, cb, sizeof(s.codebook));
    s.round_mode = round_mode;
    s.zero_floor = zero_floor ? 1 : 0;

    int nthr;
    s.thr[0] = -INFINITY;
    if (round_mode == AW4_RTN) {
        nthr = 15;
        const int64_t lo_key = fkey(-1.0f), hi_key = fkey(1.0f);
        if (rtn_literal(cb, -1.0f) != 0 || rtn_literal(cb, 1.0f) != 15)
            return fail(AW4_ERR_UNSUPPORTED, "RTN codes at -1 / +1 are not 0 / 15");
        for (int k = 1; k <= 15; ++k) {
            // smallest key in (lo, hi] whose code is >= k (the rule is monotone)
            int64_t lo = lo_key, hi = hi_key;
            while (hi - lo > 1) {
                const int64_t mid = lo + (hi - lo) / 2;
                if (rtn_literal(cb, keyf(mid)) >= k) hi = mid; else lo = mid;
            }
            s.thr[k] = keyf(hi);
        }
    } else {
        nthr = 16;
        for (int k = 0; k < 16; ++k) s.thr[k + 1] = std::nextafter(cb[k], INFINITY);
    }
    for (int k = nthr + 1; k < 18; ++k) s.thr[k] = INFINITY;
    // the fewest power-of-two bins for which no two thresholds are closer
    // than a bin width, so that no bin holds two
    double min_gap = INFINITY;
    for (int k = 1; k < nthr; ++k) min_gap = std::fmin(min_gap, (double)s.thr[k + 1] - s.thr[k]);
    s.lut_bins = 0;
    for (int nb = 32; nb <= AW4_LUT_BINS; nb *= 2)
        if (min_gap > 2.0 / nb) {
            s.lut_bins = nb;
            break;
        }
    if (s.lut_bins == 0)
        return fail(AW4_ERR_UNSUPPORTED, "codebook levels too close for the search table");
    const float half = (float)(s.lut_bins / 2);
    for (int b = 0; b < s.lut_bins; ++b) {
        const float edge = -1.0f + (float)b / half;  // exact
        int count = 0;
        for (int k = 1; k <= nthr; ++k) count += (s.thr[k] <= edge) ? 1 : 0;
        s.lut[b] = (uint8_t)count;
    }
    // verify the table against the literal rule around every threshold and
    // bin edge, and on a deterministic spread of values
    for (int k = 1; k <= nthr; ++k) {
        const int64_t c = fkey(s.thr[k]);
        for (int64_t d = -64; d <= 64; ++d) {
            const float x = keyf(c + d);
            if (x < -1.0f || x > 1.0f) continue;
            if (lut_search(s, x) != expected(s, x))
                return fail(AW4_ERR_UNSUPPORTED, "search table mismatch near threshold %d", k);
        }
    }
    for (int b = 0; b <= s.lut_bins; ++b) {
        const int64_t c = fkey(-1.0f + (float)b / half);
        for (int64_t d = -8; d <= 8; ++d) {
            const float x = keyf(c + d);
            if (x < -1.0f || x > 1.0f) continue;
            if (lut_search(s, x) != expected(s, x))
                return fail(AW4_ERR_UNSUPPORTED, "search table mismatch near bin %d", b);
        }
    }
    uint64_t st = 0x9E3779B97F4A7C15ull;
    for (int n = 0; n < (1 << 18); ++n) {
        st ^= st << 13; st ^= st >> 7; st ^= st << 17;
        const float x = bitsf((uint32_t)st);
        if (!(x >= -1.0f && x <= 1.0f)) continue;
        if (lut_search(s, x) != expected(s, x))
            return fail(AW4_ERR_UNSUPPORTED, "search table mismatch at sampled value");
    }
    // state of an all-zero moment (adamw.py:524-545)
    int zc;
    if (round_mode == AW4_RTN) {
        zc = rtn_literal(cb, 0.0f);
    } else {
        const int i = searchsorted_left(cb, 0.0f);
        const int l = i - 1 < 0 ? 0 : i - 1, r = i > 15 ? 15 : i;
        if (round_mode == AW4_SR_VALUE) {
            const float width = cb[r] - cb[l];
            float p = width > 0.0f ? (0.0f - cb[l]) / width : 0.0f;
            if (!(p == 0.0f || p == 1.0f))
                return fail(AW4_ERR_UNSUPPORTED, "zero is not an exact level of the SR codebook");
            zc = p == 1.0f ? r : l;
        } else {
            if (l != r && cb[l] != 0.0f && cb[r] != 0.0f)
                return fail(AW4_ERR_UNSUPPORTED, "zero is not an exact level of the SR codebook");
            zc = (cb[l] == 0.0f) ? l : r;
        }
    }
    if (zero_floor && zc == 0) zc = 1;
    s.zero_code = (uint8_t)zc;
    s.zero_scale = 1e-12f;
    {
        volatile float den = 0.0f * cb[zc];
        volatile float corr = 0.0f / (den < 1e-12f ? 1e-12f : den);
        s.zero_scale_eden = 1e-12f * corr;
    }
    *out = s;
    return AW4_OK;
}
