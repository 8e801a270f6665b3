/* trc_oracle.c -- TEST INFRASTRUCTURE: CPU restatement of train.cpp's quantized-weight hot path.
 * See trc_oracle.h for the function-by-function map to the reference sources. Not product code.
 *
 * Compiled with -ffp-contract=off and no -march flag: the reference's x86-64 build performs
 * every multiply and add as a separately rounded fp32 operation, and so does this file.
 */
#include "trc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <string.h>

static float f_from_bits(uint32_t w) { float f; memcpy(&f, &w, 4); return f; }
static uint32_t bits_from_f(float f) { uint32_t w; memcpy(&w, &f, 4); return w; }

/* IEEE-754 binary16 -> binary32, exact for every finite input. A NaN keeps its payload and comes
 * out quiet, which is what the reference's arithmetic decode yields on x86 (trc_float.h:23-40). */
float oracle_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t expo = (h >> 10) & 0x1Fu;
    uint32_t       mant = h & 0x3FFu;
    uint32_t       out;
    if (expo == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            /* subnormal: value = mant * 2^-24; normalise into an fp32 normal */
            int e = 113; /* 127 - 15 + 1 */
            while ((mant & 0x400u) == 0) {
                mant <<= 1;
                --e;
            }
            out = sign | ((uint32_t) e << 23) | ((mant & 0x3FFu) << 13);
        }
    } else if (expo == 0x1F) {
        out = sign | 0x7F800000u | (mant << 13);
        if (mant != 0) out |= 0x00400000u;
    } else {
        out = sign | ((expo + 112u) << 23) | (mant << 13);
    }
    return f_from_bits(out);
}

/* binary32 -> binary16, round to nearest, ties to even. */
uint16_t oracle_fp32_to_fp16(float f) {
    const uint32_t x    = bits_from_f(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax   = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return (uint16_t) (sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    if (ax >= 0x477FF000u) return (uint16_t) (sign | 0x7C00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                      /* below 2^-14: subnormal half */
        if (ax <= 0x33000000u) return (uint16_t) sign;           /* <= 2^-25 ties to zero */
        const uint32_t e     = ax >> 23;
        const uint32_t m     = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e; /* 14..24 */
        uint32_t       q     = m >> shift;
        const uint32_t rem   = m & ((1u << shift) - 1u);
        const uint32_t half  = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t) (sign | q);
    }
    uint32_t       q   = (((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q; /* a carry into the exponent is right */
    return (uint16_t) (sign | q);
}

size_t oracle_block_bytes(int type) {
    switch (type) {
        case ORACLE_Q4_0: return 18;
        case ORACLE_Q4_1: return 20;
        case ORACLE_Q5_0: return 22;
        case ORACLE_Q5_1: return 24;
        case ORACLE_Q8_0: return 34;
        default: return 0;
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t) (p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) {
    return (uint32_t) p[0] | ((uint32_t) p[1] << 8) | ((uint32_t) p[2] << 16) | ((uint32_t) p[3] << 24);
}

/* Block layouts (little-endian), 32 weights each:
 *   Q4_0 [d:f16][qs:16]          w[j] = (lo(qs[j]) - 8) d,  w[j+16] = (hi(qs[j]) - 8) d
 *   Q4_1 [d][m][qs:16]           w = q d + m
 *   Q5_0 [d][qh:u32][qs:16]      5th bit of w[j] is qh bit j, of w[j+16] is qh bit j+16; (q-16) d
 *   Q5_1 [d][m][qh][qs:16]       w = q d + m
 *   Q8_0 [d][qs:int8 x 32]       w = q d                          (trc_gguf.cpp:320-417) */
int oracle_dequant(int type, const uint8_t* src, int64_t n_blocks, float* out) {
    const size_t bb = oracle_block_bytes(type);
    if (bb == 0) return -1;
    for (int64_t blk = 0; blk < n_blocks; ++blk) {
        const uint8_t* p = src + (size_t) blk * bb;
        float*         y = out + blk * 32;
        const float    d = oracle_fp16_to_fp32(rd16(p));
        switch (type) {
            case ORACLE_Q4_0:
                for (int j = 0; j < 16; ++j) {
                    y[j]      = (float) ((p[2 + j] & 0x0F) - 8) * d;
                    y[j + 16] = (float) ((p[2 + j] >> 4) - 8) * d;
                }
                break;
            case ORACLE_Q4_1: {
                const float m = oracle_fp16_to_fp32(rd16(p + 2));
                for (int j = 0; j < 16; ++j) {
                    y[j]      = (float) (p[4 + j] & 0x0F) * d + m;
                    y[j + 16] = (float) (p[4 + j] >> 4) * d + m;
                }
            } break;
            case ORACLE_Q5_0: {
                const uint32_t qh = rd32(p + 2);
                for (int j = 0; j < 16; ++j) {
                    const int lo = (p[6 + j] & 0x0F) | (int) (((qh >> j) & 1u) << 4);
                    const int hi = (p[6 + j] >> 4) | (int) (((qh >> (j + 16)) & 1u) << 4);
                    y[j]      = (float) (lo - 16) * d;
                    y[j + 16] = (float) (hi - 16) * d;
                }
            } break;
            case ORACLE_Q5_1: {
                const float    m  = oracle_fp16_to_fp32(rd16(p + 2));
                const uint32_t qh = rd32(p + 4);
                for (int j = 0; j < 16; ++j) {
                    const int lo = (p[8 + j] & 0x0F) | (int) (((qh >> j) & 1u) << 4);
                    const int hi = (p[8 + j] >> 4) | (int) (((qh >> (j + 16)) & 1u) << 4);
                    y[j]      = (float) lo * d + m;
                    y[j + 16] = (float) hi * d + m;
                }
            } break;
            case ORACLE_Q8_0:
                for (int j = 0; j < 32; ++j) y[j] = (float) (int8_t) p[2 + j] * d;
                break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ strided F32 helpers */

static float ld(const void* base, size_t off) {
    float v;
    memcpy(&v, (const uint8_t*) base + off, 4);
    return v;
}
static void st(void* base, size_t off, float v) { memcpy((uint8_t*) base + off, &v, 4); }

typedef struct {
    const void *a, *b;
    void*       d;
    const int64_t *a_ne, *b_ne, *d_ne;
    const size_t *a_nb, *b_nb, *d_nb;
    int64_t j0, j1; /* output-column range handled by this worker */
} mm_job;

static void* mm_worker(void* arg) {
    const mm_job* J = (const mm_job*) arg;
    const int64_t k = J->a_ne[0], m = J->a_ne[1];
    for (int64_t i3 = 0; i3 < J->b_ne[3]; ++i3) {
        for (int64_t i2 = 0; i2 < J->b_ne[2]; ++i2) {
            const size_t oa = (size_t) (i2 % J->a_ne[2]) * J->a_nb[2] + (size_t) (i3 % J->a_ne[3]) * J->a_nb[3];
            const size_t ob = (size_t) i2 * J->b_nb[2] + (size_t) i3 * J->b_nb[3];
            const size_t od = (size_t) i2 * J->d_nb[2] + (size_t) i3 * J->d_nb[3];
            for (int64_t j = J->j0; j < J->j1; ++j) {
                for (int64_t i = 0; i < m; ++i) {
                    float sum = 0.0f;
                    for (int64_t kk = 0; kk < k; ++kk) {
                        sum += ld(J->a, oa + (size_t) i * J->a_nb[1] + (size_t) kk * J->a_nb[0]) *
                               ld(J->b, ob + (size_t) j * J->b_nb[1] + (size_t) kk * J->b_nb[0]);
                    }
                    st(J->d, od + (size_t) i * J->d_nb[0] + (size_t) j * J->d_nb[1], sum);
                }
            }
        }
    }
    return NULL;
}

int oracle_mul_mat(const void* a, const int64_t a_ne[4], const size_t a_nb[4],
                   const void* b, const int64_t b_ne[4], const size_t b_nb[4],
                   void* d, const int64_t d_ne[4], const size_t d_nb[4], int n_threads) {
    /* shape rules of the mul_mat constructor (trc_ops.cpp:366-385) */
    if (a_ne[0] != b_ne[0]) return -1;
    if (b_ne[2] % a_ne[2] != 0 || b_ne[3] % a_ne[3] != 0) return -1;
    if (d_ne[0] != a_ne[1] || d_ne[1] != b_ne[1] || d_ne[2] != b_ne[2] || d_ne[3] != b_ne[3]) return -1;
    const int64_t n = b_ne[1];
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_threads > n) n_threads = (int) (n > 0 ? n : 1);
    mm_job    jobs[256];
    pthread_t tids[256];
    for (int t = 0; t < n_threads; ++t) {
        mm_job* J = &jobs[t];
        J->a = a; J->b = b; J->d = d;
        J->a_ne = a_ne; J->b_ne = b_ne; J->d_ne = d_ne;
        J->a_nb = a_nb; J->b_nb = b_nb; J->d_nb = d_nb;
        J->j0 = n * t / n_threads;
        J->j1 = n * (t + 1) / n_threads;
    }
    if (n_threads == 1) {
        mm_worker(&jobs[0]);
        return 0;
    }
    for (int t = 0; t < n_threads; ++t) pthread_create(&tids[t], NULL, mm_worker, &jobs[t]);
    for (int t = 0; t < n_threads; ++t) pthread_join(tids[t], NULL);
    return 0;
}

/* linear index (i0 fastest) -> byte offset in a strided view (trc_tensor.cpp tensor_offset_linear) */
static size_t lin_off(int64_t i, const int64_t ne[4], const size_t nb[4]) {
    size_t off = 0;
    for (int dd = 0; dd < 4; ++dd) {
        off += (size_t) (i % ne[dd]) * nb[dd];
        i /= ne[dd];
    }
    return off;
}

void oracle_cont(const void* a, const int64_t a_ne[4], const size_t a_nb[4], float* dst) {
    const int64_t n = a_ne[0] * a_ne[1] * a_ne[2] * a_ne[3];
    for (int64_t i = 0; i < n; ++i) dst[i] = ld(a, lin_off(i, a_ne, a_nb));
}

void oracle_repeat_back(const void* a, const int64_t a_ne[4], const size_t a_nb[4],
                        float* dst, const int64_t dst_ne[4]) {
    const int64_t nd = dst_ne[0] * dst_ne[1] * dst_ne[2] * dst_ne[3];
    for (int64_t i = 0; i < nd; ++i) dst[i] = 0.0f;
    const int64_t n = a_ne[0] * a_ne[1] * a_ne[2] * a_ne[3];
    for (int64_t i = 0; i < n; ++i) {
        int64_t rem = i, od = 0, mul = 1;
        for (int dd = 0; dd < 4; ++dd) {
            const int64_t idx = rem % a_ne[dd];
            rem /= a_ne[dd];
            od += (idx % dst_ne[dd]) * mul;
            mul *= dst_ne[dd];
        }
        dst[od] = dst[od] + ld(a, lin_off(i, a_ne, a_nb));
    }
}

void oracle_acc(void* dst, const void* b, const int64_t b_ne[4], const size_t b_nb[4],
                size_t nb1, size_t nb2, size_t nb3, size_t offset) {
    const int64_t n = b_ne[0] * b_ne[1] * b_ne[2] * b_ne[3];
    for (int64_t i = 0; i < n; ++i) {
        int64_t rem = i, idx[4];
        for (int dd = 0; dd < 4; ++dd) {
            idx[dd] = rem % b_ne[dd];
            rem /= b_ne[dd];
        }
        const size_t od = offset + (size_t) idx[0] * 4 + (size_t) idx[1] * nb1 + (size_t) idx[2] * nb2 +
                          (size_t) idx[3] * nb3;
        st(dst, od, ld(dst, od) + ld(b, lin_off(i, b_ne, b_nb)));
    }
}

/* ---------------------------------------------------------------- the rest of a training step
 * Built with -ffp-contract=off: every operation below is one IEEE single (or double) operation in
 * the order the reference writes it, as the reference's own x86 build evaluates it. */

/* fn_neg / fn_abs / fn_sqr / fn_sqrt / fn_sgn / fn_step (src/backends/cpu/trc_cpu_ops.cpp:84-94)
 * applied by compute_unary (:119-137); compute_scale (:139-149). */
void oracle_unary(int op, const float* x, int64_t n, float param, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        float r;
        switch (op) {
            case 0: r = v * v; break;
            case 1: r = sqrtf(v); break;
            case 2: r = fabsf(v); break;
            case 3: r = -v; break;
            case 4: r = v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f); break;
            case 5: r = v > 0.0f ? 1.0f : 0.0f; break;
            default: r = v * param; break;
        }
        out[i] = r;
    }
}

/* row_sum_f32 (src/backends/cpu/trc_cpu_ops.cpp:284-300) + compute_sum_rows_or_mean (:317-333). */
void oracle_sum_rows(const float* x, int64_t ne0, int64_t rows, int take_mean, float* out) {
    for (int64_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        for (int64_t i = 0; i < ne0; ++i) sum += x[r * ne0 + i];
        out[r] = take_mean ? (float) (sum / (double) ne0) : (float) sum;
    }
}

/* compute_opt_step_adamw (src/backends/cpu/trc_cpu_ops.cpp:1506-1538). */
void oracle_adamw(float* p, const float* g, float* m, float* v, int64_t n, const float ps[6]) {
    const float step_sz = ps[0], bc2_sqrt = ps[1], decay = ps[2], beta1 = ps[3], beta2 = ps[4], eps = ps[5];
    for (int64_t i = 0; i < n; ++i) {
        const float gi = g[i];
        m[i] += (gi - m[i]) * (1.0f - beta1);
        v[i] = v[i] * beta2 + gi * gi * (1.0f - beta2);
        const float pv    = p[i] * decay;
        const float denom = sqrtf(v[i]) / bc2_sqrt + eps;
        p[i]              = pv - step_sz * (m[i] / denom);
    }
}

/* compute_opt_step_sgd (src/backends/cpu/trc_cpu_ops.cpp:1540-1573). */
void oracle_sgd(float* p, const float* g, float* mom, int64_t n, const float ps[6]) {
    const float lr = ps[0], mc = ps[1], damp = ps[2], wd = ps[3], nesterov = ps[4], is_first = ps[5];
    for (int64_t i = 0; i < n; ++i) {
        float d = g[i] + wd * p[i];
        if (mc != 0.0f) {
            if (is_first != 0.0f) mom[i] = d;
            else mom[i] = mc * mom[i] + (1.0f - damp) * d;
            d = nesterov != 0.0f ? d + mc * mom[i] : mom[i];
        }
        p[i] -= lr * d;
    }
}

/* compute_sum_sqr_acc (src/backends/cpu/trc_cpu_ops.cpp:1578-1591). */
void oracle_sum_sqr_acc(float* acc, const float* x, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double) x[i] * (double) x[i];
    acc[0] = acc[0] + (float) s;
}

/* compute_clip_scale_inplace (src/backends/cpu/trc_cpu_ops.cpp:1594-1611). */
void oracle_clip_scale(float* x, int64_t n, float norm, float max_norm, float eps) {
    const float total = sqrtf(norm);
    float scale = max_norm / (total + eps);
    if (scale > 1.0f) scale = 1.0f;
    for (int64_t i = 0; i < n; ++i) x[i] *= scale;
}
