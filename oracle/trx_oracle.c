/*
 * trx_oracle.c -- C restatement of the TriXium engine matvec.  TEST INFRASTRUCTURE ONLY:
 * the checker and the timed CPU baseline ("port") of bench.py; never on the product path.
 *
 * Restates, on the converter's packed row packets:
 *   - row-packet geometry      model/layout.py:189-217
 *   - code decode              model/bons.py:125-130 (trit5, digit k of byte i = lane 5i+k),
 *                              model/bons.py:188-190 (2-bit, code j at bits 2*(j%4) of byte j/4)
 *   - fp16 decomposition       model/bitexact.py:56-68
 *   - engine matvec            model/bitexact.py:101-119 (int64 accumulate, floor shifts,
 *                              overflow checks of :116 and :118)
 *   - quantiser                model/mirror.py:34-51 (floor(x+0.5) in fp32, e8 = frexp - 7)
 *   - float projection         model/mirror.py:648-678 (int32 result * 2^(e8+R-B))
 *   - fp projection            model/fastref.py:103-125 (fp32 sum of (code-1)*x per group
 *                              times the scale; summation order differs from BLAS)
 * Rows are independent: OpenMP splits them over the host's threads.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static uint8_t DIG[256][5];
static int dig_ready = 0;

static void init_digits(void) {
    if (dig_ready) return;
    for (int b = 0; b < 256; ++b) {
        int v = b;
        for (int k = 0; k < 5; ++k) {
            DIG[b][k] = (uint8_t)(v % 3);
            v /= 3;
        }
    }
    dig_ready = 1;
}

int trxo_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void trxo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

long trxo_row_bytes(int cols, int kind) {
    long G = cols / 128;
    long sb = (G + 15) / 16 * 32;
    long cb = kind == 5 ? 26 * G : 32 * G;
    return sb + (cb + 31) / 32 * 32;
}

static void fp16_split(uint16_t u, int64_t *m11, int *e16) {
    int E = (u >> 10) & 31;
    int64_t m = E ? (int64_t)((u & 1023) | 1024) : (int64_t)(u & 1023);
    *m11 = (u & 0x8000) ? -m : m;
    *e16 = E ? E - 25 : -24;
}

/* Digits of one group into codes[128]. */
static void group_codes(const uint8_t *cb, int kind, uint8_t *codes) {
    if (kind == 5) {
        for (int i = 0; i < 26; ++i)
            for (int k = 0; k < 5; ++k) {
                int l = 5 * i + k;
                if (l < 128) codes[l] = DIG[cb[i]][k];
            }
    } else {
        for (int l = 0; l < 128; ++l) codes[l] = (cb[l >> 2] >> (2 * (l & 3))) & 3;
    }
}

/* Integer engine matvec; returns the number of rows that overflowed (0 = ok). */
int trxo_matvec_int(const uint8_t *packed, int rows, int cols, int kind, const int8_t *x8, int B, int R,
                    int32_t *out) {
    init_digits();
    const int G = cols / 128;
    const long rb = trxo_row_bytes(cols, kind);
    const long sb = (G + 15) / 16 * 32;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = packed + (long)r * rb;
        int64_t acc = 0;
        uint8_t codes[128];
        for (int g = 0; g < G; ++g) {
            const uint8_t *cb = row + sb + (kind == 5 ? 26L * g : 32L * g);
            group_codes(cb, kind, codes);
            int64_t gs = 0;
            for (int l = 0; l < 128; ++l) gs += (int64_t)((int)codes[l] - 1) * x8[g * 128 + l];
            uint16_t sbits;
            memcpy(&sbits, row + 2 * g, 2);
            int64_t m11;
            int e16;
            fp16_split(sbits, &m11, &e16);
            int64_t prod = gs * m11;
            int sh = e16 + B;
            acc += sh >= 0 ? prod * ((int64_t)1 << (sh > 62 ? 62 : sh)) : prod >> (-sh > 63 ? 63 : -sh);
        }
        int64_t res = acc >> R;
        if (acc >= ((int64_t)1 << 47) || acc <= -((int64_t)1 << 47) || res >= ((int64_t)1 << 31) ||
            res <= -((int64_t)1 << 31))
            bad += 1;
        out[r] = (int32_t)res;
    }
    return bad;
}

static int lround_mirror(float x) {
    volatile float t;
    if (x >= 0.f) {
        t = x + 0.5f;
        return (int)floorf(t);
    }
    t = x - 0.5f;
    return (int)ceilf(t);
}

/* Power-of-two int8 quantiser; returns e8. */
int trxo_quantize(const float *x, int n, int8_t *x8) {
    float amax = 0.f;
    for (int i = 0; i < n; ++i) {
        float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    if (amax == 0.f) {
        memset(x8, 0, (size_t)n);
        return 0;
    }
    int e;
    frexpf(amax, &e);
    const int e8 = e - 7;
    const float inv = ldexpf(1.0f, -e8);
    for (int i = 0; i < n; ++i) {
        int q = lround_mirror(x[i] * inv);
        x8[i] = (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
    }
    return e8;
}

/* Float projection in the engine's arithmetic; x8 is caller scratch of cols bytes. */
int trxo_matvec_f(const uint8_t *packed, int rows, int cols, int kind, int B, int R, const float *x, float *y,
                  int8_t *x8, int32_t *scratch) {
    const int e8 = trxo_quantize(x, cols, x8);
    const int bad = trxo_matvec_int(packed, rows, cols, kind, x8, B, R, scratch);
    const float sc = ldexpf(1.0f, e8 + R - B);
    for (int r = 0; r < rows; ++r) y[r] = (float)scratch[r] * sc;
    return bad;
}

/* fp-mode projection. */
void trxo_matvec_fp(const uint8_t *packed, int rows, int cols, int kind, const float *x, float *y) {
    init_digits();
    const int G = cols / 128;
    const long rb = trxo_row_bytes(cols, kind);
    const long sb = (G + 15) / 16 * 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = packed + (long)r * rb;
        uint8_t codes[128];
        float acc = 0.f;
        for (int g = 0; g < G; ++g) {
            group_codes(row + sb + (kind == 5 ? 26L * g : 32L * g), kind, codes);
            float s = 0.f;
            for (int l = 0; l < 128; ++l) s += (float)((int)codes[l] - 1) * x[g * 128 + l];
            uint16_t sbits;
            memcpy(&sbits, row + 2 * g, 2);
            /* fp16 -> fp32 exactly: m11 * 2^e16 */
            int64_t m11;
            int e16;
            fp16_split(sbits, &m11, &e16);
            acc += s * ldexpf((float)m11, e16);
        }
        y[r] = acc;
    }
}
