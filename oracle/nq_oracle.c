/*
 * CPU oracle for the NanoQuant quantized-linear path.  TEST INFRASTRUCTURE ONLY:
 * this file is the checker that tests, the smoke entry point and the CPU baseline
 * leg of the benchmark compare the CUDA path against.  Nothing in the product
 * (nanoquant_b200/) links, loads or calls it.
 *
 * It restates, in plain C, the reference algorithm of rkuznetsovcg/NanoQuant:
 *   - nqo_pack    : src/nanoquant/kernel/utils.py:51-113   (pack_binary_gemv)
 *   - nqo_unpack  : src/nanoquant/kernel/utils.py:116-183  (unpack_binary_gemv)
 *   - nqo_forward : src/nanoquant/modules/linear.py:282-291 (_compute_forward),
 *                   evaluated in double precision on the packed sign planes.
 *
 * Bit conventions (utils.py:87-106): a sign of +1 maps to bit 0 and -1 to bit 1;
 * rows are padded with +1 up to a multiple of 32 columns; column j of a 32-column
 * chunk lands on bit j ("lsb_first", order 0) or on bit 15 - j/2 + 16*(j%2)
 * ("half2", order 1).
 *
 * Validity: the reference packer computes (1 - s) // 2 and so silently produces
 * carries for values other than +-1; nqo_pack instead reports the number of
 * entries that are not exactly +-1 through its return value (the reference
 * module rejects such factors before packing, linear.py:369-370).
 */
#include <stdint.h>
#include <stddef.h>

#define NQO_LSB_FIRST 0
#define NQO_HALF2 1

static int nqo_bitpos(int j, int order) {
    if (order == NQO_LSB_FIRST) return j;
    return 15 - j / 2 + 16 * (j % 2);
}

/* Returns the number of entries that are not exactly +1 or -1, or -1 for a bad order. */
long nqo_pack(const int8_t *signs, long rows, long cols, int order, int32_t *out) {
    if (order != NQO_LSB_FIRST && order != NQO_HALF2) return -1;
    long words = (cols + 31) / 32;
    long bad = 0;
    for (long r = 0; r < rows; ++r) {
        for (long w = 0; w < words; ++w) {
            uint32_t word = 0;
            for (int j = 0; j < 32; ++j) {
                long c = w * 32 + j;
                int bit = 0; /* padding columns are +1 -> bit 0 */
                if (c < cols) {
                    int8_t s = signs[r * cols + c];
                    if (s != 1 && s != -1) ++bad;
                    bit = s < 0;
                }
                word |= (uint32_t)bit << nqo_bitpos(j, order);
            }
            out[r * words + w] = (int32_t)word;
        }
    }
    return bad;
}

int nqo_unpack(const int32_t *packed, long rows, long cols, int order, int8_t *out) {
    if (order != NQO_LSB_FIRST && order != NQO_HALF2) return -1;
    long words = (cols + 31) / 32;
    for (long r = 0; r < rows; ++r) {
        for (long c = 0; c < cols; ++c) {
            uint32_t word = (uint32_t)packed[r * words + c / 32];
            int bit = (word >> nqo_bitpos((int)(c % 32), order)) & 1;
            out[r * cols + c] = (int8_t)(1 - 2 * bit);
        }
    }
    return 0;
}

static inline double nqo_sign(const int32_t *plane, long words, long row, long col, int order) {
    uint32_t word = (uint32_t)plane[row * words + col / 32];
    return ((word >> nqo_bitpos((int)(col % 32), order)) & 1) ? -1.0 : 1.0;
}

/*
 * y[b, m] = s1[m] * sum_k U[m, k] * smid[k] * sum_n V[k, n] * s2[n] * x[b, n]
 * x: [batch, in]; v_bits: [rank, ceil(in/32)]; u_bits: [out, ceil(rank/32)];
 * smid may be NULL (no scale_mid, the plain nanoquant export).  interm (optional,
 * may be NULL) receives smid * (V (s2 . x)) as [batch, rank].
 */
int nqo_forward(const float *x, long batch, long in_f, const float *s2, const int32_t *v_bits,
                long rank, const float *smid, const int32_t *u_bits, long out_f,
                const float *s1, int order, double *y, double *interm) {
    if (order != NQO_LSB_FIRST && order != NQO_HALF2) return -1;
    long wv = (in_f + 31) / 32, wu = (rank + 31) / 32;
    for (long b = 0; b < batch; ++b) {
        const float *xb = x + b * in_f;
        /* stage 1: t[k] = smid[k] * sum_n V[k, n] * (s2[n] * x[n]) */
        double *t = interm ? interm + b * rank : NULL;
        for (long m = 0; m < out_f; ++m) y[b * out_f + m] = 0.0;
        for (long k = 0; k < rank; ++k) {
            double acc = 0.0;
            for (long n = 0; n < in_f; ++n)
                acc += nqo_sign(v_bits, wv, k, n, order) * ((double)s2[n] * (double)xb[n]);
            if (smid) acc *= (double)smid[k];
            if (t) t[k] = acc;
            /* stage 2 accumulated column by column: y[m] += U[m, k] * t[k] */
            for (long m = 0; m < out_f; ++m)
                y[b * out_f + m] += nqo_sign(u_bits, wu, m, k, order) * acc;
        }
        for (long m = 0; m < out_f; ++m) y[b * out_f + m] *= (double)s1[m];
    }
    return 0;
}
