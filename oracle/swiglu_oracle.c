/*
 * CPU oracle for the batch-one SwiGLU decode layer -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this
 * library, and only as the checker. The CUDA product path never calls it.
 *
 * Plain-C restatement of shubhxho/cuda-kernel's host contract; every function
 * names the reference lines it follows. Build with -ffp-contract=off so float
 * expressions round exactly as the reference's x86-64 host build rounds them.
 */
#include "swiglu_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    const int e = (int)(ax >> 23) - 127;
    const uint32_t m = ax & 0x7fffffu;
    if (e >= -14) { /* normal binary16 */
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        const uint32_t rem = m & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may bump the exponent */
        return (uint16_t)(sign | h);
    }
    if (e < -25 - 1) return sign; /* far below half the smallest subnormal */
    /* subnormal: value = sig * 2^(e-23); in units of 2^-24 that is sig * 2^(e+1) */
    const uint32_t sig = (e == -127) ? m : (m | 0x800000u);
    const int shift = -(e + 1);
    if (shift > 31) return sign;
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1f) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else { /* subnormal half: normalise */
        int k = 0;
        while (!(m & 0x400u)) { m <<= 1; ++k; }
        m &= 0x3ffu;
        bits = sign | ((uint32_t)(113 - k) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static float g_f16_table[65536];

__attribute__((constructor)) static void orc_init_table(void) {
    for (uint32_t i = 0; i < 65536u; ++i) g_f16_table[i] = orc_f16_to_f32((uint16_t)i);
}

void orc_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(in[i]);
}

void orc_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = g_f16_table[in[i]];
}

/* ------------------------------------------------------------ contract */

/* contract.hpp:21 -- two branches keep exp() from overflowing. */
double orc_silu(double x) {
    if (x >= 0) return x / (1.0 + exp(-x));
    const double e = exp(x);
    return x * e / (1.0 + e);
}

/* contract.hpp:23-34 -- row-major, one double accumulator per row, columns in order. */
int orc_matvec(const float* w, const float* x, int rows, int cols, float* y) {
    if (rows <= 0 || cols <= 0 || !w || !x || !y) return ORC_EINVAL;
    for (int r = 0; r < rows; ++r) {
        const float* wr = w + (size_t)r * (size_t)cols;
        double sum = 0;
        for (int c = 0; c < cols; ++c) sum += (double)wr[c] * (double)x[c];
        y[r] = (float)sum;
    }
    return ORC_OK;
}

int orc_matvec_f16(const uint16_t* w, const float* x, int rows, int cols, float* y) {
    if (rows <= 0 || cols <= 0 || !w || !x || !y) return ORC_EINVAL;
    for (int r = 0; r < rows; ++r) {
        const uint16_t* wr = w + (size_t)r * (size_t)cols;
        double sum = 0;
        for (int c = 0; c < cols; ++c) sum += (double)g_f16_table[wr[c]] * (double)x[c];
        y[r] = (float)sum;
    }
    return ORC_OK;
}

/* contract.hpp:36-53 */
int orc_compare(const float* actual, const float* expected, size_t n, double atol, double rtol,
                double* max_abs, double* max_scaled, int* passed) {
    if (n == 0 || !actual || !expected) return ORC_EINVAL;
    if (!isfinite(atol) || !isfinite(rtol) || atol <= 0 || rtol < 0) return ORC_EINVAL;
    double ma = 0, ms = 0;
    int ok = 1;
    for (size_t i = 0; i < n; ++i) {
        if (!isfinite(actual[i]) || !isfinite(expected[i])) {
            ok = 0;
            ma = ms = INFINITY;
            continue;
        }
        const double delta = fabs((double)actual[i] - (double)expected[i]);
        const double scaled = delta / (atol + rtol * fabs((double)expected[i]));
        if (delta > ma) ma = delta;
        if (scaled > ms) ms = scaled;
        ok &= scaled <= 1.0;
    }
    if (max_abs) *max_abs = ma;
    if (max_scaled) *max_scaled = ms;
    if (passed) *passed = ok;
    return ORC_OK;
}

static int cmp_double(const void* a, const void* b) {
    const double x = *(const double*)a, y = *(const double*)b;
    return (x > y) - (x < y);
}

/* contract.hpp:54-60 */
int orc_median(const double* xs, size_t n, double* out) {
    if (n == 0 || !xs || !out) return ORC_EINVAL;
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(xs[i]) || xs[i] <= 0) return ORC_EINVAL;
    double* s = (double*)malloc(n * sizeof *s);
    if (!s) return ORC_EINVAL;
    memcpy(s, xs, n * sizeof *s);
    qsort(s, n, sizeof *s, cmp_double);
    *out = (n % 2) ? s[n / 2] : (s[n / 2 - 1] + s[n / 2]) / 2;
    free(s);
    return ORC_OK;
}

/* contract.hpp:61-71 */
size_t orc_json_escape(const char* in, char* out, size_t cap) {
    static const char hex[] = "0123456789abcdef";
    size_t k = 0;
#define ORC_PUT(ch)                       \
    do {                                  \
        if (out && k + 1 < cap) out[k] = (ch); \
        ++k;                              \
    } while (0)
    for (const unsigned char* p = (const unsigned char*)in; *p; ++p) {
        const unsigned char c = *p;
        if (c == '"' || c == '\\') {
            ORC_PUT('\\');
            ORC_PUT((char)c);
        } else if (c < 32) {
            ORC_PUT('\\'); ORC_PUT('u'); ORC_PUT('0'); ORC_PUT('0');
            ORC_PUT(hex[c >> 4]);
            ORC_PUT(hex[c & 15]);
        } else {
            ORC_PUT((char)c);
        }
    }
#undef ORC_PUT
    if (out && cap) out[k < cap ? k : cap - 1] = '\0';
    return k;
}

/* ----------------------------------------------------------------- FFN */

/* benchmark.cu:131-141, in the same order and precision. */
int orc_ffn(const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, const uint16_t* x,
            const uint16_t* bg, const uint16_t* bu, const uint16_t* bd, int hidden, int inter,
            float* proj, uint16_t* act, float* y) {
    if (hidden <= 0 || inter <= 0 || !wg || !wu || !wd || !x || !bg || !bu || !bd || !y) return ORC_EINVAL;
    float* fx = (float*)malloc((size_t)hidden * sizeof *fx);
    float* g = (float*)malloc((size_t)inter * sizeof *g);
    float* u = (float*)malloc((size_t)inter * sizeof *u);
    float* a = (float*)malloc((size_t)inter * sizeof *a);
    int rc = ORC_EINVAL;
    if (!fx || !g || !u || !a) goto done;
    orc_f16_to_f32_array(x, fx, (size_t)hidden);
    orc_matvec_f16(wg, fx, inter, hidden, g);
    orc_matvec_f16(wu, fx, inter, hidden, u);
    for (int i = 0; i < inter; ++i) {
        const double v = orc_silu((double)g[i] + (double)g_f16_table[bg[i]]) *
                         ((double)u[i] + (double)g_f16_table[bu[i]]);
        const uint16_t hb = orc_f32_to_f16((float)v);
        a[i] = g_f16_table[hb];
        if (act) act[i] = hb;
    }
    orc_matvec_f16(wd, a, hidden, inter, y); /* matvec(Wd, activation) */
    for (int i = 0; i < hidden; ++i) {
        const float xb = fx[i] + g_f16_table[bd[i]];
        y[i] = y[i] + xb;
    }
    if (proj) memcpy(proj, g, (size_t)inter * sizeof *g);
    rc = ORC_OK;
done:
    free(fx);
    free(g);
    free(u);
    free(a);
    return rc;
}

static inline float round16(float v) { return g_f16_table[orc_f32_to_f16(v)]; }

/* kernels.cuh:98-107 gate epilogue. Without model rounding it uses the FFN
 * reference's double-precision activation (benchmark.cu:136-138). */
int orc_gate(const uint16_t* wg, const uint16_t* wu, const uint16_t* x, const uint16_t* bg,
             const uint16_t* bu, int rows, int cols, int model_round, uint16_t* h) {
    if (rows <= 0 || cols <= 0 || !wg || !wu || !x || !h) return ORC_EINVAL;
    float* fx = (float*)malloc((size_t)cols * sizeof *fx);
    float* g = (float*)malloc((size_t)rows * sizeof *g);
    float* u = (float*)malloc((size_t)rows * sizeof *u);
    int rc = ORC_EINVAL;
    if (!fx || !g || !u) goto done;
    orc_f16_to_f32_array(x, fx, (size_t)cols);
    orc_matvec_f16(wg, fx, rows, cols, g);
    orc_matvec_f16(wu, fx, rows, cols, u);
    for (int i = 0; i < rows; ++i) {
        if (model_round) {
            float a = g[i], b = u[i];
            if (bg) a = a + g_f16_table[bg[i]];
            if (bu) b = b + g_f16_table[bu[i]];
            a = round16(a);
            b = round16(b);
            const float s = round16((float)orc_silu((double)a));
            h[i] = orc_f32_to_f16(s * b);
        } else {
            const double v = orc_silu((double)g[i] + (bg ? (double)g_f16_table[bg[i]] : 0.0)) *
                             ((double)u[i] + (bu ? (double)g_f16_table[bu[i]] : 0.0));
            h[i] = orc_f32_to_f16((float)v);
        }
    }
    rc = ORC_OK;
done:
    free(fx);
    free(g);
    free(u);
    return rc;
}

/* kernels.cuh:98-99,108-111 plain epilogue: a += bias; a += residual; fp32 or fp16 out. */
int orc_project(const uint16_t* w, const uint16_t* x, const uint16_t* bias, const uint16_t* residual,
                int rows, int cols, float* y, uint16_t* yh) {
    if (rows <= 0 || cols <= 0 || !w || !x || (!y && !yh)) return ORC_EINVAL;
    float* fx = (float*)malloc((size_t)cols * sizeof *fx);
    float* a = (float*)malloc((size_t)rows * sizeof *a);
    int rc = ORC_EINVAL;
    if (!fx || !a) goto done;
    orc_f16_to_f32_array(x, fx, (size_t)cols);
    orc_matvec_f16(w, fx, rows, cols, a);
    for (int i = 0; i < rows; ++i) {
        float v = a[i];
        if (bias) v = v + g_f16_table[bias[i]];
        if (residual) v = v + g_f16_table[residual[i]];
        if (y) y[i] = v;
        if (yh) yh[i] = orc_f32_to_f16(v);
    }
    rc = ORC_OK;
done:
    free(fx);
    free(a);
    return rc;
}

/* torch_extension.cu:34-38: model-rounding gate, then half-output down (no bias, no residual). */
int orc_ffn_model(const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, const uint16_t* x,
                  int hidden, int inter, uint16_t* h, uint16_t* y) {
    if (hidden <= 0 || inter <= 0 || !h || !y) return ORC_EINVAL;
    int rc = orc_gate(wg, wu, x, NULL, NULL, inter, hidden, 1, h);
    if (rc) return rc;
    return orc_project(wd, h, NULL, NULL, hidden, inter, NULL, y);
}

/* --------------------------------------------------------- generation */

/* MT19937 initialisation and tempering as published by Matsumoto & Nishimura. */
void orc_mt_seed(orc_mt19937* s, uint32_t seed) {
    s->mt[0] = seed;
    for (uint32_t i = 1; i < 624; ++i) s->mt[i] = 1812433253u * (s->mt[i - 1] ^ (s->mt[i - 1] >> 30)) + i;
    s->idx = 624;
}

uint32_t orc_mt_next(orc_mt19937* s) {
    if (s->idx >= 624) {
        for (int i = 0; i < 624; ++i) {
            const uint32_t y = (s->mt[i] & 0x80000000u) | (s->mt[(i + 1) % 624] & 0x7fffffffu);
            s->mt[i] = s->mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        s->idx = 0;
    }
    uint32_t y = s->mt[s->idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* benchmark.cu:89-94. libstdc++ draws a float in [0,1) from one 32-bit output
 * (generate_canonical<float,24>: float(u) / 2^32, clamped below 1) and maps it
 * with (b - a) * r + a, each step rounded to float. */
void orc_random_half(orc_mt19937* s, size_t n, float scale, uint16_t* out) {
    const float a = -scale, b = scale;
    const float width = b - a;
    for (size_t i = 0; i < n; ++i) {
        const float sum = (float)orc_mt_next(s);
        float r = sum / 4294967296.0f;
        if (r >= 1.0f) r = nextafterf(1.0f, 0.0f);
        const float prod = r * width;
        const float v = prod + a;
        out[i] = orc_f32_to_f16(v);
    }
}

/* benchmark.cu:116-121 */
int orc_reference_workload(uint32_t seed, int hidden, int inter, uint16_t* wg, uint16_t* wu,
                           uint16_t* wd, uint16_t* x, uint16_t* bg, uint16_t* bu, uint16_t* bd) {
    if (hidden <= 0 || inter <= 0 || !wg || !wu || !wd || !x || !bg || !bu || !bd) return ORC_EINVAL;
    orc_mt19937 s;
    orc_mt_seed(&s, seed);
    const size_t n = (size_t)hidden * (size_t)inter;
    orc_random_half(&s, n, 1.0f / sqrtf((float)hidden), wg);
    orc_random_half(&s, n, 1.0f / sqrtf((float)hidden), wu);
    orc_random_half(&s, n, 1.0f / sqrtf((float)inter), wd);
    orc_random_half(&s, (size_t)hidden, 1.0f, x);
    orc_random_half(&s, (size_t)inter, 0.1f, bg);
    orc_random_half(&s, (size_t)inter, 0.1f, bu);
    orc_random_half(&s, (size_t)hidden, 0.1f, bd);
    return ORC_OK;
}
