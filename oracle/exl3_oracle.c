/*
 * EXL3 CPU oracle -- TEST INFRASTRUCTURE ONLY (see exl3_oracle.h).
 *
 * Restates, in plain C, the algorithm of the reference project
 * jyohukuchan/xiaomi-hexagon-exl3; each function cites the file:line it
 * follows.  Used by tests/, __graft_entry__.smoke() and bench.py's CPU leg as
 * the checker; never by the shipped CUDA library.
 */
#include "exl3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp16 <-> fp32, IEEE round-to-nearest-even (src/exl3_codec.cpp:21-66) ---- */

float orc_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp5 = (h >> 10) & 0x1fu;
    const uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    float out;
    if (exp5 == 0) {
        /* zero or subnormal: mant * 2^-24, exact in fp32 */
        float mag = ldexpf((float)mant, -24);
        return (h & 0x8000u) ? -mag : mag;
    }
    if (exp5 == 31) bits = sign | 0x7f800000u | (mant << 13);
    else bits = sign | ((exp5 + 112u) << 23) | (mant << 13);
    memcpy(&out, &bits, 4);
    return out;
}

/* value >> shift, rounded to nearest with ties to even */
static uint32_t shr_rne(uint32_t value, unsigned shift) {
    const uint32_t kept = value >> shift;
    const uint32_t rest = value & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    return kept + ((rest > half) || (rest == half && (kept & 1u)));
}

uint16_t orc_float_to_half(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const uint32_t exp8 = (bits >> 23) & 0xffu;
    const uint32_t mant = bits & 0x7fffffu;
    if (exp8 == 0xffu) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u)); /* inf / canonical qNaN */
    if (exp8 >= 143u) return (uint16_t)(sign | 0x7c00u);                    /* >= 2^16 overflows */
    if (exp8 <= 101u) return sign;                                          /* < 2^-25 rounds to zero */
    if (exp8 <= 112u) return (uint16_t)(sign | shr_rne(mant | 0x800000u, 126u - exp8)); /* subnormal */
    /* normal; a mantissa carry legitimately bumps the exponent (65520 -> inf) */
    return (uint16_t)(sign | (((exp8 - 112u) << 10) + shr_rne(mant, 13u)));
}

/* ---- state -> fp16 codebooks (src/exl3_codec.cpp:68-86) ---- */

uint16_t orc_decode_codebook(uint16_t state, unsigned codebook) {
    uint32_t p = state;
    if (codebook == ORC_CB_MUL1) {
        /* byte sum of state * 0x83dcd12d, mapped through 0x6400+s -> fp16(1024+s),
           then one fused multiply-add by fp16 0x1eee and 0xc931 */
        p *= 0x83dcd12du;
        const unsigned s = (p & 0xffu) + ((p >> 8) & 0xffu) + ((p >> 16) & 0xffu) + (p >> 24);
        const float base = orc_half_to_float((uint16_t)(0x6400u + s));
        return orc_float_to_half(fmaf(base, orc_half_to_float(0x1eeeu), orc_half_to_float(0xc931u)));
    }
    if (codebook == ORC_CB_MCG) p *= 0xcbac1fedu;
    else p = p * 89226354u + 64248484u; /* 3inst */
    p = (p & 0x8fff8fffu) ^ 0x3b603b60u;
    return orc_float_to_half(orc_half_to_float((uint16_t)p) + orc_half_to_float((uint16_t)(p >> 16)));
}

static uint16_t g_tables[3][65536];
static pthread_once_t g_tables_once = PTHREAD_ONCE_INIT;

static void build_tables(void) {
    for (unsigned cb = 0; cb < 3; ++cb)
        for (unsigned s = 0; s < 65536u; ++s) g_tables[cb][s] = orc_decode_codebook((uint16_t)s, cb);
}

static int valid_codec(unsigned bits, unsigned codebook) { return bits >= 1 && bits <= 8 && codebook <= 2; }

/* ---- trellis tile (src/exl3_codec.cpp:88-115) ----
 * A tile is 16*bits uint16 = 8*bits 32-bit words, word i = u16[2i] | u16[2i+1] << 16,
 * read as one big-endian bit ring of 256*bits bits.  Position p's state is the
 * 16-bit window that ends at ring bit (p+1)*bits (tail-biting), and it lands at
 * row (L%4)*2 + (e&1) + 8*(e>>1&1), column L/4 + 8*(e>>2) with L = p/8, e = p%8. */
static uint32_t ring_word(const uint16_t * packed, unsigned i) {
    return (uint32_t)packed[2 * i] | ((uint32_t)packed[2 * i + 1] << 16);
}

static void tile_states(const uint16_t * packed, unsigned bits, uint16_t states[256]) {
    const unsigned ring = 256u * bits;
    for (unsigned p = 0; p < 256u; ++p) {
        const unsigned end = ((p + 1u) * bits) % ring;         /* window end, exclusive */
        const unsigned first = (end + ring - 16u) % ring;      /* window start */
        const unsigned last = (end + ring - 1u) % ring;        /* final bit of the window */
        const uint64_t hi = ring_word(packed, first / 32u);
        const uint64_t lo = ring_word(packed, last / 32u);
        const unsigned drop = 31u - (last % 32u);
        uint64_t both = (first / 32u == last / 32u) ? lo : ((hi << 32) | lo);
        states[p] = (uint16_t)(both >> drop);
    }
}

static void tile_place(const uint16_t states[256], const uint16_t * table, uint16_t * row_major) {
    for (unsigned p = 0; p < 256u; ++p) {
        const unsigned L = p >> 3, e = p & 7u;
        const unsigned row = (L & 3u) * 2u + (e & 1u) + ((e & 2u) << 2);
        const unsigned col = (L >> 2) + ((e & 4u) << 1);
        row_major[row * 16u + col] = table[states[p]];
    }
}

int orc_decode_tile(const uint16_t * packed, unsigned bits, unsigned codebook, uint16_t * tile256) {
    uint16_t states[256];
    if (!valid_codec(bits, codebook)) return 1;
    pthread_once(&g_tables_once, build_tables);
    tile_states(packed, bits, states);
    tile_place(states, g_tables[codebook], tile256);
    return 0;
}

/* ---- inner matrix and column slices (src/exl3_codec.cpp:117-145) ---- */

static int valid_shape(size_t k, size_t n, size_t multiple) {
    return k && n && !(k % multiple) && !(n % multiple) && k <= ((size_t)-1) / n;
}

int orc_decode_inner(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                     unsigned bits, unsigned codebook, uint16_t * out) {
    uint16_t tile[256];
    if (!valid_codec(bits, codebook) || !valid_shape(k, n, 16)) return 1;
    if (!column_count || first_column % 16 || column_count % 16 || first_column > n ||
        column_count > n - first_column) return 1;
    for (size_t rk = 0; rk < k / 16; ++rk) {
        for (size_t cn = 0; cn < column_count / 16; ++cn) {
            const uint16_t * src = packed + (rk * (n / 16) + first_column / 16 + cn) * 16u * bits;
            orc_decode_tile(src, bits, codebook, tile);
            for (size_t r = 0; r < 16; ++r)
                memcpy(out + (rk * 16 + r) * column_count + cn * 16, tile + r * 16, 32);
        }
    }
    return 0;
}

/* ---- orthonormal Walsh-Hadamard over 128-value groups (src/exl3_codec.cpp:147-167) ----
 * butterflies with stride 1, 2, ..., 64 (a+b, a-b), then a single multiply by 1/sqrt(128) */
int orc_hadamard128(float * v, size_t count) {
    const float norm = 0.08838834764831844055f;
    if (count % 128) return 1;
    for (size_t g = 0; g < count; g += 128) {
        float * x = v + g;
        for (unsigned h = 1; h < 128u; h <<= 1) {
            for (unsigned i = 0; i < 128u; ++i) {
                if (i & h) continue;
                const float a = x[i], b = x[i + h];
                x[i] = a + b;
                x[i + h] = a - b;
            }
        }
        for (unsigned i = 0; i < 128u; ++i) x[i] *= norm;
    }
    return 0;
}

/* ---- original-basis reconstruction (src/exl3_codec.cpp:169-204) ----
 * W = diag(suh) H W_inner H diag(svh) per 128x128 block: rows of the block are
 * rotated first, then columns, then both scales applied and rounded to fp16. */
int orc_reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                    size_t first_column, size_t column_count, unsigned bits, unsigned codebook, uint16_t * out) {
    float * block;
    float col[128];
    if (!valid_shape(k, n, 128) || first_column % 128 || column_count % 128) return 1;
    if (orc_decode_inner(packed, k, n, first_column, column_count, bits, codebook, out)) return 1;
    block = (float *)malloc(sizeof(float) * 128 * 128);
    if (!block) return 1;
    for (size_t rk = 0; rk < k; rk += 128) {
        for (size_t cn = 0; cn < column_count; cn += 128) {
            for (size_t r = 0; r < 128; ++r)
                for (size_t c = 0; c < 128; ++c)
                    block[r * 128 + c] = orc_half_to_float(out[(rk + r) * column_count + cn + c]);
            orc_hadamard128(block, 128 * 128);
            for (size_t c = 0; c < 128; ++c) {
                for (size_t r = 0; r < 128; ++r) col[r] = block[r * 128 + c];
                orc_hadamard128(col, 128);
                for (size_t r = 0; r < 128; ++r) {
                    const float val = col[r] * orc_half_to_float(suh[rk + r]) *
                                      orc_half_to_float(svh[first_column + cn + c]);
                    out[(rk + r) * column_count + cn + c] = orc_float_to_half(val);
                }
            }
        }
    }
    free(block);
    return 0;
}

/* ---- runtime group records (include/exl3-block.h:14,34-39; tools/export_native_gguf.py:27-36) ----
 * record (nb,kb) at index nb*(k/128)+kb: 64 tiles in order r*8+c (r = 16-row
 * sub-tile, c = 16-column sub-tile), each 32*bits bytes; then suh[kb*128..+128],
 * then svh[nb*128..+128] as fp16. */
size_t orc_group_bytes(unsigned bits) { return 2048u * bits + 512u; }

int orc_pack_records(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                     unsigned bits, uint8_t * records) {
    const size_t tile_bytes = 32u * bits;
    if (bits < 1 || bits > 8 || !valid_shape(k, n, 128)) return 1;
    for (size_t nb = 0; nb < n / 128; ++nb) {
        for (size_t kb = 0; kb < k / 128; ++kb) {
            uint8_t * rec = records + (nb * (k / 128) + kb) * orc_group_bytes(bits);
            for (size_t r = 0; r < 8; ++r)
                for (size_t c = 0; c < 8; ++c) {
                    const uint16_t * src = packed + ((kb * 8 + r) * (n / 16) + nb * 8 + c) * 16u * bits;
                    memcpy(rec + (r * 8 + c) * tile_bytes, src, tile_bytes);
                }
            memcpy(rec + 2048u * bits, suh + kb * 128, 256);
            memcpy(rec + 2048u * bits + 256u, svh + nb * 128, 256);
        }
    }
    return 0;
}

/* ---- CPU operator (src/exl3-ggml.cpp:51-92) ---- */

struct mm_job {
    const uint8_t * records;
    unsigned bits, codebook;
    size_t k, n, rows, y_stride;
    const float * xh;
    float * y;
    int ith, nth;
};

static void * mm_worker(void * arg) {
    const struct mm_job * j = (const struct mm_job *)arg;
    const size_t gb = orc_group_bytes(j->bits);
    const size_t kblocks = j->k / 128;
    float * acc = (float *)calloc(j->rows * 128, sizeof(float));
    uint16_t * w = (uint16_t *)malloc(128 * 128 * sizeof(uint16_t));
    float * wf = (float *)malloc(128 * 128 * sizeof(float));
    if (!acc || !w || !wf) abort();
    for (size_t nb = (size_t)j->ith; nb < j->n / 128; nb += (size_t)j->nth) {
        memset(acc, 0, j->rows * 128 * sizeof(float));
        for (size_t kb = 0; kb < kblocks; ++kb) {
            const uint8_t * rec = j->records + (nb * kblocks + kb) * gb;
            orc_decode_inner((const uint16_t *)rec, 128, 128, 0, 128, j->bits, j->codebook, w);
            for (size_t t = 0; t < 128 * 128; ++t) wf[t] = orc_half_to_float(w[t]);
            for (size_t i = 0; i < 128; ++i)
                for (size_t c = 0; c < 128; ++c) {
                    const float wv = wf[i * 128 + c];
                    for (size_t r = 0; r < j->rows; ++r) acc[r * 128 + c] += j->xh[r * j->k + kb * 128 + i] * wv;
                }
        }
        {
            const uint16_t * sv = (const uint16_t *)(j->records + nb * kblocks * gb + 2048u * j->bits + 256u);
            for (size_t r = 0; r < j->rows; ++r) {
                orc_hadamard128(acc + r * 128, 128);
                for (size_t c = 0; c < 128; ++c)
                    j->y[r * j->y_stride + nb * 128 + c] = acc[r * 128 + c] * orc_half_to_float(sv[c]);
            }
        }
    }
    free(acc);
    free(w);
    free(wf);
    return NULL;
}

int orc_mul_mat(const uint8_t * records, unsigned bits, unsigned codebook, size_t k, size_t n, const void * x,
                int x_is_f16, size_t rows, size_t x_stride, float * y, size_t y_stride, int nth) {
    const size_t gb = orc_group_bytes(bits);
    float * xh;
    if (!valid_codec(bits, codebook) || !valid_shape(k, n, 128) || !rows) return 1;
    if (nth < 1) nth = 1;
    pthread_once(&g_tables_once, build_tables);
    /* phase 1: xh = H128(x * su) per row and 128-block; su comes from record (0,kb) */
    xh = (float *)malloc(rows * k * sizeof(float));
    if (!xh) return 1;
    for (size_t kb = 0; kb < k / 128; ++kb) {
        const uint16_t * su = (const uint16_t *)(records + kb * gb + 2048u * bits);
        for (size_t r = 0; r < rows; ++r) {
            for (size_t c = 0; c < 128; ++c) {
                const size_t at = r * x_stride + kb * 128 + c;
                const float v = x_is_f16 ? orc_half_to_float(((const uint16_t *)x)[at]) : ((const float *)x)[at];
                xh[r * k + kb * 128 + c] = v * orc_half_to_float(su[c]);
            }
            orc_hadamard128(xh + r * k + kb * 128, 128);
        }
    }
    /* phases 2-3 on nth threads over output column blocks */
    {
        struct mm_job * jobs = (struct mm_job *)calloc((size_t)nth, sizeof(struct mm_job));
        pthread_t * tids = (pthread_t *)calloc((size_t)nth, sizeof(pthread_t));
        if (!jobs || !tids) abort();
        for (int t = 0; t < nth; ++t) {
            struct mm_job jb = {records, bits, codebook, k, n, rows, y_stride, xh, y, t, nth};
            jobs[t] = jb;
            if (t) pthread_create(&tids[t], NULL, mm_worker, &jobs[t]);
        }
        mm_worker(&jobs[0]);
        for (int t = 1; t < nth; ++t) pthread_join(tids[t], NULL);
        free(jobs);
        free(tids);
    }
    free(xh);
    return 0;
}

/* ---- tied-head embedding lookup (src/exl3-ggml.cpp:19-49) ----
 * for each id and each 128-row block kb: reconstruct group (id/128, kb) in the
 * original basis and take column id%128. */
int orc_get_rows(const uint8_t * records, unsigned bits, unsigned codebook, size_t k, size_t n, const int32_t * ids,
                 size_t count, float * out) {
    const size_t gb = orc_group_bytes(bits);
    uint16_t * block;
    if (!valid_codec(bits, codebook) || !valid_shape(k, n, 128)) return 1;
    for (size_t i = 0; i < count; ++i)
        if (ids[i] < 0 || (size_t)ids[i] >= n) return 1;
    block = (uint16_t *)malloc(128 * 128 * sizeof(uint16_t));
    if (!block) return 1;
    for (size_t i = 0; i < count; ++i) {
        const size_t id = (size_t)ids[i];
        for (size_t kb = 0; kb < k / 128; ++kb) {
            const uint8_t * rec = records + ((id / 128) * (k / 128) + kb) * gb;
            orc_reconstruct((const uint16_t *)rec, (const uint16_t *)(rec + 2048u * bits),
                            (const uint16_t *)(rec + 2048u * bits + 256u), 128, 128, 0, 128, bits, codebook, block);
            for (size_t r = 0; r < 128; ++r) out[i * k + kb * 128 + r] = orc_half_to_float(block[r * 128 + id % 128]);
        }
    }
    free(block);
    return 0;
}
