/*
 * C restatement of the reference's CPU dequantize + GEMV path.
 * TEST INFRASTRUCTURE ONLY: used by tests/ as a full-size checker and by the
 * CPU-baseline leg of bench.py as the reference CPU path being timed. The
 * product library never links or loads it.
 *
 * Reference (KrishnaI2424/Dequant_Project):
 *   dequant/packer.py:164-174  unpack      slot s of a word holds logical code
 *                                          order[s] at bits [b*s, b*s+b)
 *   dequant/packer.py:177-189  dequantize  fp16((q - off) * scale), fp32 math
 *   dequant/packer.py:37-41    _INTERLEAVE slot orders
 *   F.linear(x, packer.dequantize(pw)) is the CPU GEMV path the reference's
 *   kernel is judged against (scripts/test_quant_linear.py:306-321).
 *
 * oracle_dequantize is bit-exact with packer.dequantize. oracle_gemv computes
 * y[m,n] = fp16( sum_k float(x[m,k]) * float(Wdeq[n,k]) ) with Wdeq the fp16
 * dequantized weight and an fp32 accumulator, i.e. the arithmetic of torch's
 * CPU F.linear on fp16 operands up to summation order.
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef _Float16 half_t;

static const int ORDER4[8] = {0, 2, 4, 6, 1, 3, 5, 7};
static const int ORDER2[16] = {0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15};
static const int ORDER8[4] = {0, 2, 1, 3};

static float h2f(uint16_t h) {
    half_t v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static uint16_t f2h(float f) {
    half_t v = (half_t)f; /* IEEE round-to-nearest-even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static const int *slot_order(int bits, int interleaved) {
    if (!interleaved) return NULL;
    return bits == 4 ? ORDER4 : (bits == 2 ? ORDER2 : ORDER8);
}

/* Dequantize one row into fp16-rounded floats (the values packer.dequantize
 * stores), following dequant/packer.py:177-189. A word never straddles a
 * group because group_size is a multiple of the codes per word. */
static void dequant_row(const uint32_t *qrow, const uint16_t *srow, const uint16_t *zrow,
                        float *out, int K, int bits, int gs, int symmetric,
                        const int *order) {
    const int per = 32 / bits;
    const uint32_t qmax = (1u << bits) - 1u;
    const float bias = (float)(1 << (bits - 1));
    const int words = K / per;
    for (int w = 0; w < words; ++w) {
        const uint32_t word = qrow[w];
        const int k0 = w * per;
        const int g = k0 / gs;
        const float off = symmetric ? bias : h2f(zrow[g]);
        const float scale = h2f(srow[g]);
        for (int s = 0; s < per; ++s) {
            const int logical = order ? order[s] : s;
            const float q = (float)((word >> (bits * s)) & qmax);
            out[k0 + logical] = h2f(f2h((q - off) * scale));
        }
    }
}

/* fp32 dot product with 16 independent partial sums (vectorisable without
 * reassociation flags); the summation order differs from torch's anyway. */
static float dot16(const float *a, const float *b, int K) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= K; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += a[k + j] * b[k + j];
    float s = 0.f;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; k < K; ++k) s += a[k] * b[k];
    return s;
}

int oracle_dequantize(const int32_t *qweight, const uint16_t *scales, const uint16_t *zeros,
                      uint16_t *out, int N, int K, int bits, int group_size, int symmetric,
                      int interleaved, int nthreads) {
    if (bits != 2 && bits != 4 && bits != 8) return 1;
    if (group_size <= 0 || K % group_size || group_size % (32 / bits)) return 2;
    const int G = K / group_size;
    const int *order = slot_order(bits, interleaved);
    int err = 0;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)K);
        if (!row) {
#pragma omp atomic write
            err = 3;
        } else {
#pragma omp for schedule(static)
            for (int n = 0; n < N; ++n) {
                dequant_row((const uint32_t *)qweight + (size_t)n * (K / (32 / bits)),
                            scales + (size_t)n * G, zeros ? zeros + (size_t)n * G : NULL,
                            row, K, bits, group_size, symmetric, order);
                uint16_t *o = out + (size_t)n * K;
                for (int k = 0; k < K; ++k) o[k] = f2h(row[k]);
            }
            free(row);
        }
    }
    return err;
}

int oracle_gemv(const uint16_t *x, int M, const int32_t *qweight, const uint16_t *scales,
                const uint16_t *zeros, uint16_t *y, int N, int K, int bits, int group_size,
                int symmetric, int interleaved, int nthreads) {
    if (bits != 2 && bits != 4 && bits != 8) return 1;
    if (group_size <= 0 || K % group_size || group_size % (32 / bits)) return 2;
    if (M < 1) return 4;
    const int G = K / group_size;
    const int *order = slot_order(bits, interleaved);
    float *xf = (float *)malloc(sizeof(float) * (size_t)M * K);
    if (!xf) return 3;
    for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = h2f(x[i]);
    int err = 0;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)K);
        if (!row) {
#pragma omp atomic write
            err = 3;
        } else {
#pragma omp for schedule(static)
            for (int n = 0; n < N; ++n) {
                dequant_row((const uint32_t *)qweight + (size_t)n * (K / (32 / bits)),
                            scales + (size_t)n * G, zeros ? zeros + (size_t)n * G : NULL,
                            row, K, bits, group_size, symmetric, order);
                for (int m = 0; m < M; ++m) {
                    y[(size_t)m * N + n] = f2h(dot16(xf + (size_t)m * K, row, K));
                }
            }
            free(row);
        }
    }
    free(xf);
    return err;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
