/*
 * CPU oracle for the NVFP4 paged KV-cache path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's Triton kernels
 * (Plaaasma/glm53-flash-dual-dgx-spark, nvfp4-kv/glm53_nvfp4_runtime.py) so the CUDA
 * kernels of this repository can be checked bit for bit.  It is linked only by tests/,
 * __graft_entry__.smoke() and the cpu_baseline / reference arm of bench.py; the product
 * path never calls it.
 *
 * Parity pin: the golden fixtures in tests/golden/ were produced by running the
 * reference's own _quant_kernel / _gather_kernel through the Triton interpreter (with
 * its fp32<->fp8 conversion replaced by torch's IEEE round-to-nearest-even cast, because
 * the interpreter's own conversion rounds ties away from zero); tests/test_oracle.py
 * checks this file against them.
 *
 * Semantics that the reference leaves to the hardware and that are fixed here:
 *   - fp32 division is IEEE round-to-nearest (the interpreter's numpy semantics);
 *   - fp32 -> e4m3 is round-to-nearest-even with saturation to +-448 (cvt.rn.satfinite);
 *   - max() ignores NaN operands (fmaxf), as Triton's maximum does on the GPU.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define NV_BYTES 288
#define DS_BYTES 656
#define LATENT 512

/* ---------------------------------------------------------------- number formats */

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static float f16_to_f32(uint16_t h) {
    uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 31u, m = h & 1023u;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | 1024u), (int)e - 25);
    return (float)(s ? -v : v);
}

/* e4m3 (fn variant: bias 7, no infinities, S.1111.111 = NaN) -> fp32, exact. */
float oracle_e4m3_to_f32(uint8_t b) {
    uint32_t s = b >> 7, e = (b >> 3) & 15u, m = b & 7u;
    double v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexp((double)m, -9);
    else v = ldexp((double)(m | 8u), (int)e - 10);
    return (float)(s ? -v : v);
}

/* fp32 -> e4m3, round to nearest even, saturating finite values to +-448.  A NaN input
 * gives the canonical NaN byte 0x7f whatever its sign bit: GPU arithmetic produces the
 * canonical (positive) fp32 NaN, so a NaN never carries a sign into the conversion there.
 * Written from the format definition; all intermediate arithmetic is exact in double. */
uint8_t oracle_f32_to_e4m3(float x) {
    if (isnan(x)) return 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    double a = fabs((double)x);
    if (a >= 448.0) return (uint8_t)(sign | 0x7e);
    if (a < ldexp(1.0, -6)) {                       /* subnormal range: k * 2^-9 */
        double k = nearbyint(a * 512.0);            /* default rounding mode: to nearest even */
        return (uint8_t)(sign | (uint8_t)k);        /* k == 8 encodes 2^-6, the first normal */
    }
    int e;
    double fr = frexp(a, &e);                       /* a = fr * 2^e, fr in [0.5, 1) */
    int ex = e - 1;                                 /* a = 1.m * 2^ex */
    double mant = nearbyint((fr * 2.0 - 1.0) * 8.0);
    if (mant >= 8.0) { mant = 0.0; ex += 1; }
    int be = ex + 7;
    if (be > 15 || (be == 15 && mant >= 7.0)) return (uint8_t)(sign | 0x7e);
    return (uint8_t)(sign | (uint8_t)(be << 3) | (uint8_t)mant);
}

/* e2m1 magnitude code (3 bits) -> value, following _e2m1 (glm53_nvfp4_runtime.py:81-85). */
static float e2m1_mag(uint32_t mag) {
    uint32_t e = mag >> 1, m = mag & 1u;
    if (e == 0) return 0.5f * (float)m;
    return ldexpf(1.0f + 0.5f * (float)m, (int)e - 1);
}

/* Threshold ladder of _quant_kernel (glm53_nvfp4_runtime.py:57-64); a NaN quotient fails
 * every `<` and lands on 7, exactly like the chained tl.where. */
static uint32_t ladder(float v) {
    float a = fabsf(v);
    uint32_t c;
    if (a < 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a < 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a < 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a < 5.0f) c = 6;
    else c = 7;
    return c | (v < 0.0f ? 8u : 0u);
}

/* ---------------------------------------------------------------- append */

/* One token: 512 values -> one 288-byte pool row.
 * Follows _quant_kernel (glm53_nvfp4_runtime.py:37-65). */
void oracle_quant_row(const float* x, uint8_t* row) {
    float s[32];
    for (int g = 0; g < 32; ++g) {
        float amax = 0.0f;
        int any = 0;
        for (int i = 0; i < 16; ++i) {
            float a = fabsf(x[16 * g + i]);
            if (!any) { amax = a; any = 1; } else amax = fmaxf(amax, a);
        }
        float sc = fmaxf(amax / 6.0f, 1e-8f);                 /* :47 */
        uint8_t sb = oracle_f32_to_e4m3(sc);
        row[256 + g] = sb;                                     /* :48 */
        s[g] = oracle_e4m3_to_f32(sb);                         /* :49 */
    }
    for (int i = 0; i < 256; ++i) {                            /* :51-65 */
        float si = s[i / 8];
        float lo = x[2 * i] / si;
        float hi = x[2 * i + 1] / si;
        row[i] = (uint8_t)(ladder(lo) | (ladder(hi) << 4));
    }
}

/* kv_c: T rows of 512 elements (bf16 if dtype==0, fp16 if dtype==1) with a row stride
 * of `stride` elements; rows whose slot is negative are skipped (:42-43). */
void oracle_quant_rows(const uint16_t* kv_c, int dtype, int64_t T, int64_t stride,
                       uint8_t* pool, int64_t pool_rows, const int64_t* slot) {
    float x[LATENT];
    for (int64_t t = 0; t < T; ++t) {
        int64_t sl = slot[t];
        if (sl < 0 || sl >= pool_rows) continue;
        const uint16_t* src = kv_c + t * stride;
        for (int i = 0; i < LATENT; ++i)
            x[i] = dtype == 0 ? bf16_to_f32(src[i]) : f16_to_f32(src[i]);
        oracle_quant_row(x, pool + sl * NV_BYTES);
    }
}

/* ---------------------------------------------------------------- dequant */

/* Pool row -> 512 fp32 values (code value times its block scale; exact in fp32). */
void oracle_dequant_row(const uint8_t* row, float* out) {
    for (int b = 0; b < 256; ++b) {
        uint32_t byte = row[b];
        uint32_t lo_c = byte & 15u, hi_c = byte >> 4;
        float s16 = oracle_e4m3_to_f32(row[256 + (2 * b) / 16]);
        /* The reference negates with Triton's unary minus, which lowers to `0 - x`: the
         * code 0x8 therefore decodes to +0.0, and a zero takes its sign from the scale. */
        float lo = (lo_c & 8u) ? 0.0f - e2m1_mag(lo_c & 7u) : e2m1_mag(lo_c & 7u);
        float hi = (hi_c & 8u) ? 0.0f - e2m1_mag(hi_c & 7u) : e2m1_mag(hi_c & 7u);
        out[2 * b] = lo * s16;
        out[2 * b + 1] = hi * s16;
    }
}

/* rows[i] < 0 or >= pool_rows produce a zero row. */
void oracle_dequant_rows(const uint8_t* pool, int64_t pool_rows, const int64_t* rows,
                         int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        int64_t r = rows[i];
        if (r < 0 || r >= pool_rows) { memset(out + i * LATENT, 0, LATENT * sizeof(float)); continue; }
        oracle_dequant_row(pool + r * NV_BYTES, out + i * LATENT);
    }
}

/* ---------------------------------------------------------------- 656-byte gather */

/* Follows _gather_kernel (glm53_nvfp4_runtime.py:87-122): one gathered NVFP4 row becomes
 * one fp8_ds_mla row: 512 e4m3 bytes, four fp32 per-128 scales, 128 zero bytes. */
void oracle_gather_ds656(const uint8_t* pool, int64_t pool_rows, const int32_t* idx,
                         int64_t S, uint8_t* out) {
    float v[LATENT];
    for (int64_t r = 0; r < S; ++r) {
        int64_t src = idx[r];
        if (src < 0) src = 0;                                  /* :98 clamp */
        if (src > pool_rows - 1) src = pool_rows - 1;
        oracle_dequant_row(pool + src * NV_BYTES, v);          /* :99-108 */
        uint8_t* o = out + r * DS_BYTES;
        for (int j = 0; j < 4; ++j) {                          /* :109-114 */
            float amax = 0.0f;
            for (int b = 64 * j; b < 64 * j + 64; ++b) {
                float m = fmaxf(fabsf(v[2 * b]), fabsf(v[2 * b + 1]));
                amax = fmaxf(amax, m);
            }
            float gscale = fmaxf(amax / 448.0f, 1e-12f);
            memcpy(o + 512 + 4 * j, &gscale, 4);
            float inv = 1.0f / gscale;                         /* :115-116 */
            for (int b = 64 * j; b < 64 * j + 64; ++b) {       /* :117-120 */
                o[2 * b] = oracle_f32_to_e4m3(v[2 * b] * inv);
                o[2 * b + 1] = oracle_f32_to_e4m3(v[2 * b + 1] * inv);
            }
        }
        memset(o + 528, 0, 128);                               /* :121-122 */
    }
}

/* ---------------------------------------------------------------- batched helpers */

/* Vectorised conversions used by the Python side of the oracle. */
void oracle_f32_to_e4m3_array(const float* x, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_e4m3(x[i]);
}

void oracle_e4m3_to_f32_array(const uint8_t* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_f32(x[i]);
}
