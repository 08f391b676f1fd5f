/*
 * vk_oracle.c — CPU oracle for the paged KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the reference
 * VULCAN algorithms that the CUDA library replaces, so that tests, the smoke
 * check and the CPU baseline of the benchmark can check or time them.  Nothing
 * in the product library links or calls it.
 *
 * Followed reference code (paths inside the VULCAN project):
 *   - cpu_attention           tests/test_attention.cu:53-103   (golden attention)
 *   - KVCache::append         src/kv_cache.cpp:84-128          (row scatter)
 *   - GQA head mapping        src/transformer.cpp:173-189      (q_head = kv*G + rep)
 *   - MemoryManager pages     cuda/memory.cu:73-191            (byte pages, swap)
 *   - cpu_rope                tests/test_kernels.cu:697-716    (rotary embedding,
 *                             applied to Q and K_new at src/transformer.cpp:114-128)
 *   - group quantisation      docs/ADRs/003-quantization-format.md:11-18 (symmetric
 *                             per-group fp32 scale; FP8 pages use it with e4m3)
 *   - launch_matmul           cuda/matmul.cu:42-103            (C = A * B, the wo
 *                             projection of src/transformer.cpp:191-194)
 *
 * Floating point follows cpu_attention exactly: fp32 accumulation in the same
 * loop order, -FLT_MAX fill, max-subtracted expf, divide by the sum, then the
 * weighted V sum with the key index innermost.  Build with -ffp-contract=off
 * and without -ffast-math so that the results are bit-identical to the
 * reference's golden function compiled the same way.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* IEEE binary16 -> binary32, exact (all fp16 values are representable). */
static float or_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

void or_h2f_array(const uint16_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = or_h2f(in[i]);
}

/*
 * Full causal attention over contiguous [B, H, S, D] fp32 arrays: the
 * restatement of cpu_attention (tests/test_attention.cu:53-103).
 */
void or_attention_causal(const float* Q, const float* K, const float* V, float* O,
                         int B, int H, int S, int D) {
    const float scale = 1.0f / sqrtf((float)D);           /* :60 */
    float* scores = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    for (int b = 0; b < B; ++b) {
        for (int h = 0; h < H; ++h) {
            const int64_t bh = (int64_t)((b * H + h) * S) * D; /* :64 */
            for (int row = 0; row < S; ++row) {
                for (int j = 0; j < S; ++j) scores[j] = -FLT_MAX; /* :68 */
                for (int j = 0; j <= row; ++j) {                  /* :69-76 */
                    float dot = 0.0f;
                    for (int d = 0; d < D; ++d)
                        dot += Q[bh + (int64_t)row * D + d] * K[bh + (int64_t)j * D + d];
                    scores[j] = dot * scale;
                }
                float max_s = scores[0];                          /* :79-80 */
                for (int j = 1; j <= row; ++j)
                    if (max_s < scores[j]) max_s = scores[j];
                float sum = 0.0f;                                 /* :81-85 */
                for (int j = 0; j <= row; ++j) {
                    scores[j] = expf(scores[j] - max_s);
                    sum += scores[j];
                }
                for (int j = 0; j <= row; ++j) scores[j] /= sum;  /* :86-88 */
                for (int d = 0; d < D; ++d) {                     /* :91-97 */
                    float val = 0.0f;
                    for (int j = 0; j <= row; ++j)
                        val += scores[j] * V[bh + (int64_t)j * D + d];
                    O[bh + (int64_t)row * D + d] = val;
                }
            }
        }
    }
    free(scores);
}

/* Pool geometry (see include/vk_paged_kv.h for the layout). */
typedef struct {
    int L, Hkv, D, P, num_pages;
} or_geom;

static inline int64_t or_row_off(const or_geom* g, int64_t page, int layer, int head, int kv,
                                 int slot) {
    /* element offset of row (layer, page, head, kv, slot): layer-major pool */
    int64_t chunk = (((int64_t)layer * g->num_pages + page) * g->Hkv + head);
    return ((chunk * 2 + kv) * g->P + slot) * (int64_t)g->D;
}

/*
 * One attention row against keys 0..n-1 of a paged sequence, the arithmetic of
 * one cpu_attention row (tests/test_attention.cu:66-97) with K_j / V_j gathered
 * through the block table.  q: fp32 [D].  out: fp32 [D].  Returns 0, or -1 on
 * a bad table entry.
 */
static int or_row_paged(const or_geom* g, const uint16_t* pool, int layer, int kvh,
                        const float* q, const int32_t* bt, int bt_stride, int n, float scale,
                        float* scores, float* kbuf, float* out) {
    const int D = g->D, P = g->P;
    if (n <= 0) {
        for (int d = 0; d < D; ++d) out[d] = 0.0f;
        return 0;
    }
    if ((n + P - 1) / P > bt_stride) return -1;
    for (int j = 0; j < n; ++j) {
        int32_t page = bt[j / P];
        if (page < 0 || page >= g->num_pages) return -1;
        const uint16_t* k = pool + or_row_off(g, page, layer, kvh, 0, j % P);
        for (int d = 0; d < D; ++d) kbuf[d] = or_h2f(k[d]);
        float dot = 0.0f;
        for (int d = 0; d < D; ++d) dot += q[d] * kbuf[d];
        scores[j] = dot * scale;
    }
    float max_s = scores[0];
    for (int j = 1; j < n; ++j)
        if (max_s < scores[j]) max_s = scores[j];
    float sum = 0.0f;
    for (int j = 0; j < n; ++j) {
        scores[j] = expf(scores[j] - max_s);
        sum += scores[j];
    }
    for (int j = 0; j < n; ++j) scores[j] /= sum;
    for (int d = 0; d < D; ++d) out[d] = 0.0f;
    /* weighted V, key index innermost per output element as in :91-97 */
    for (int d = 0; d < D; ++d) {
        float val = 0.0f;
        for (int j = 0; j < n; ++j) {
            int32_t page = bt[j / P];
            const uint16_t* v = pool + or_row_off(g, page, layer, kvh, 1, j % P);
            val += scores[j] * or_h2f(v[d]);
        }
        out[d] = val;
    }
    return 0;
}

/*
 * Paged GQA decode: for every sequence b and query head h, the last causal row
 * over seq_lens[b] keys.  q: fp16 [B, Hq, D]; out: fp32 [B, Hq, D].
 * scale <= 0 selects 1/sqrtf(D).  nthreads > 1 runs (b, h) pairs in parallel
 * (each pair's arithmetic is unchanged).  Returns 0 or -1 (bad table entry).
 */
int or_decode_paged(const uint16_t* pool, int L, int Hkv, int D, int P, int num_pages,
                    int layer, const uint16_t* q, float* out, const int32_t* block_tables,
                    int bt_stride, const int32_t* seq_lens, int B, int Hq, float scale,
                    int nthreads) {
    or_geom g = {L, Hkv, D, P, num_pages};
    if (Hq % Hkv != 0) return -1;
    const int G = Hq / Hkv;
    if (scale <= 0.0f) scale = 1.0f / sqrtf((float)D);
    int max_n = 1;
    for (int b = 0; b < B; ++b)
        if (seq_lens[b] > max_n) max_n = seq_lens[b];
    int bad = 0;
    const int pairs = B * Hq;
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1) reduction(| : bad)
#endif
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)max_n);
        float* kbuf = (float*)malloc(sizeof(float) * (size_t)D);
        float* qf = (float*)malloc(sizeof(float) * (size_t)D);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int pi = 0; pi < pairs; ++pi) {
            const int b = pi / Hq, h = pi % Hq;
            const uint16_t* qh = q + ((int64_t)b * Hq + h) * D;
            for (int d = 0; d < D; ++d) qf[d] = or_h2f(qh[d]);
            if (or_row_paged(&g, pool, layer, h / G, qf, block_tables + (int64_t)b * bt_stride,
                             bt_stride, seq_lens[b], scale, scores, kbuf,
                             out + ((int64_t)b * Hq + h) * D) != 0)
                bad = 1;
        }
        free(scores);
        free(kbuf);
        free(qf);
    }
    (void)nthreads;
    return bad ? -1 : 0;
}

/*
 * Chunked prefill: query token t of sequence b at position positions[b]+t
 * attends keys 0..positions[b]+t (the causal j <= row rule of
 * tests/test_attention.cu:69).  q: fp16 [B, T, Hq, D]; out: fp32 [B, T, Hq, D].
 */
int or_prefill_paged(const uint16_t* pool, int L, int Hkv, int D, int P, int num_pages,
                     int layer, const uint16_t* q, float* out, const int32_t* block_tables,
                     int bt_stride, const int32_t* positions, int B, int T, int Hq,
                     float scale, int nthreads) {
    or_geom g = {L, Hkv, D, P, num_pages};
    if (Hq % Hkv != 0) return -1;
    const int G = Hq / Hkv;
    if (scale <= 0.0f) scale = 1.0f / sqrtf((float)D);
    int max_n = 1;
    for (int b = 0; b < B; ++b)
        if (positions[b] + T > max_n) max_n = positions[b] + T;
    int bad = 0;
    const int64_t rows = (int64_t)B * T * Hq;
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1) reduction(| : bad)
#endif
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)max_n);
        float* kbuf = (float*)malloc(sizeof(float) * (size_t)D);
        float* qf = (float*)malloc(sizeof(float) * (size_t)D);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            const int h = (int)(r % Hq);
            const int t = (int)((r / Hq) % T);
            const int b = (int)(r / ((int64_t)Hq * T));
            const uint16_t* qh = q + r * D;
            for (int d = 0; d < D; ++d) qf[d] = or_h2f(qh[d]);
            if (or_row_paged(&g, pool, layer, h / G, qf, block_tables + (int64_t)b * bt_stride,
                             bt_stride, positions[b] + t + 1, scale, scores, kbuf,
                             out + r * D) != 0)
                bad = 1;
        }
        free(scores);
        free(kbuf);
        free(qf);
    }
    (void)nthreads;
    return bad ? -1 : 0;
}

/*
 * Append: the row scatter of KVCache::append (src/kv_cache.cpp:94-121) with page
 * indirection.  k_new/v_new: fp16 [B, T, Hkv, D].  Returns 0, or -1 if a
 * position falls outside the block table or a table entry outside the pool
 * (the reference prints and returns on overflow, :87-92; nothing is written for
 * the offending token here).
 */
int or_append_paged(uint16_t* pool, int L, int Hkv, int D, int P, int num_pages, int layer,
                    const uint16_t* k_new, const uint16_t* v_new, const int32_t* block_tables,
                    int bt_stride, const int32_t* positions, int B, int T) {
    or_geom g = {L, Hkv, D, P, num_pages};
    int bad = 0;
    for (int b = 0; b < B; ++b) {
        for (int t = 0; t < T; ++t) {
            const int pos = positions[b] + t;
            if (pos < 0 || pos / P >= bt_stride) { bad = 1; continue; }
            const int32_t page = block_tables[(int64_t)b * bt_stride + pos / P];
            if (page < 0 || page >= num_pages) { bad = 1; continue; }
            for (int h = 0; h < Hkv; ++h) {
                const int64_t src = (((int64_t)b * T + t) * Hkv + h) * D;
                memcpy(pool + or_row_off(&g, page, layer, h, 0, pos % P), k_new + src,
                       sizeof(uint16_t) * (size_t)D);
                memcpy(pool + or_row_off(&g, page, layer, h, 1, pos % P), v_new + src,
                       sizeof(uint16_t) * (size_t)D);
            }
        }
    }
    return bad ? -1 : 0;
}

/* Page copy: dst_ids[i] <- src_ids[i], whole pages, applied in order.  A page
 * is nseg segments of seg_bytes; segment s of page id is at
 * s*seg_stride + id*seg_bytes (one segment per layer of a KV pool; a byte pool
 * has one segment). */
int or_copy_pages(uint8_t* pool, int nseg, uint64_t seg_bytes, uint64_t seg_stride, int num_pages,
                  const int32_t* src_ids, const int32_t* dst_ids, int n) {
    for (int i = 0; i < n; ++i) {
        if (src_ids[i] < 0 || src_ids[i] >= num_pages || dst_ids[i] < 0 ||
            dst_ids[i] >= num_pages)
            return -1;
        for (int s = 0; s < nseg; ++s)
            memmove(pool + (uint64_t)s * seg_stride + (uint64_t)dst_ids[i] * seg_bytes,
                    pool + (uint64_t)s * seg_stride + (uint64_t)src_ids[i] * seg_bytes, (size_t)seg_bytes);
    }
    return 0;
}

/* Block-table remap: entries e in [0, map_len) become page_map[e]. */
void or_remap_block_tables(int32_t* bt, int64_t entries, const int32_t* page_map, int map_len) {
    for (int64_t i = 0; i < entries; ++i)
        if (bt[i] >= 0 && bt[i] < map_len) bt[i] = page_map[bt[i]];
}

/* Double-precision decode row, to measure the fp32 oracle's own rounding. */
int or_decode_paged_f64(const uint16_t* pool, int L, int Hkv, int D, int P, int num_pages,
                        int layer, const uint16_t* q, double* out,
                        const int32_t* block_tables, int bt_stride, const int32_t* seq_lens,
                        int B, int Hq, double scale) {
    or_geom g = {L, Hkv, D, P, num_pages};
    if (Hq % Hkv != 0) return -1;
    const int G = Hq / Hkv;
    if (scale <= 0.0) scale = 1.0 / sqrt((double)D);
    for (int b = 0; b < B; ++b) {
        const int n = seq_lens[b];
        const int32_t* bt = block_tables + (int64_t)b * bt_stride;
        double* s = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
        for (int h = 0; h < Hq; ++h) {
            const uint16_t* qh = q + ((int64_t)b * Hq + h) * D;
            double* o = out + ((int64_t)b * Hq + h) * D;
            for (int d = 0; d < D; ++d) o[d] = 0.0;
            if (n <= 0) continue;
            double m = -INFINITY, sum = 0.0;
            for (int j = 0; j < n; ++j) {
                int32_t page = bt[j / P];
                if (page < 0 || page >= num_pages) { free(s); return -1; }
                const uint16_t* k = pool + or_row_off(&g, page, layer, h / G, 0, j % P);
                double dot = 0.0;
                for (int d = 0; d < D; ++d) dot += (double)or_h2f(qh[d]) * (double)or_h2f(k[d]);
                s[j] = dot * scale;
                if (s[j] > m) m = s[j];
            }
            for (int j = 0; j < n; ++j) { s[j] = exp(s[j] - m); sum += s[j]; }
            for (int j = 0; j < n; ++j) {
                const uint16_t* v = pool + or_row_off(&g, bt[j / P], layer, h / G, 1, j % P);
                for (int d = 0; d < D; ++d) o[d] += s[j] / sum * (double)or_h2f(v[d]);
            }
        }
        free(s);
    }
    return 0;
}

/* RoPE of one head_dim vector at position pos, restating cpu_rope
 * (tests/test_kernels.cu:697-716) step for step: pair i = (2i, 2i+1),
 * freq = 1 / theta_base^(2i/head_dim), angle = pos * freq,
 * (x0 cos - x1 sin, x0 sin + x1 cos).  `in` and `out` may alias. */
void or_rope(const float* in, float* out, int head_dim, int pos, float theta_base) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        const float freq = 1.0f / powf(theta_base, 2.0f * (float)i / (float)head_dim);
        const float theta = (float)pos * freq;
        const float cos_t = cosf(theta);
        const float sin_t = sinf(theta);
        const float x0 = in[2 * i];
        const float x1 = in[2 * i + 1];
        out[2 * i] = x0 * cos_t - x1 * sin_t;
        out[2 * i + 1] = x0 * sin_t + x1 * cos_t;
    }
}

/* ---- FP8 KV pages ---------------------------------------------------------
 * Restates the product's FP8 page format: the group-wise symmetric rule of
 * VULCAN's ADR-003 (docs/ADRs/003-quantization-format.md:11-18: one fp32 scale
 * per group, scale = max|group| / qmax, value = code * scale) with the OCP
 * FP8 E4M3 element (qmax 448) and the group = one token's K or V row of one
 * head.  Element codes follow the OCP 8-bit floating point definition: 1 sign,
 * 4 exponent (bias 7), 3 mantissa bits, subnormals for exponent 0, no
 * infinities, S.1111.111 = NaN, largest finite 448. */

/* Nearest-even E4M3 code of x; finite values beyond 448 saturate to +-448. */
uint8_t or_e4m3_encode(float x) {
    const uint8_t sign = signbit(x) ? 0x80 : 0x00;
    const float a = fabsf(x);
    if (isnan(x)) return (uint8_t)(sign | 0x7F);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
    if (a < 0.015625f) { /* below 2^-6: subnormal steps of 2^-9 (code 8 is 2^-6) */
        const float q = nearbyintf(a * 512.0f);
        return (uint8_t)(sign | (uint8_t)q);
    }
    int e2;
    const float f = frexpf(a, &e2); /* a = f * 2^e2, f in [0.5, 1) */
    int E = e2 - 1;                 /* a = (2f) * 2^E, 2f in [1, 2) */
    float m = nearbyintf((2.0f * f - 1.0f) * 8.0f);
    if (m >= 8.0f) {
        m = 0.0f;
        ++E;
    }
    if (E > 8 || (E == 8 && m > 6.0f)) return (uint8_t)(sign | 0x7E);
    return (uint8_t)(sign | (uint8_t)((E + 7) << 3) | (uint8_t)m);
}

float or_e4m3_decode(uint8_t c) {
    const int E = (c >> 3) & 15, m = c & 7;
    float v;
    if (E == 15 && m == 7) v = NAN;
    else if (E == 0) v = ldexpf((float)m, -9);
    else v = ldexpf(1.0f + (float)m / 8.0f, E - 7);
    return (c & 0x80) ? -v : v;
}

/* One group: amax below FLT_MIN gives scale 0 and zero codes; otherwise
 * code_i = e4m3(x_i * (448 / amax)), scale = amax / 448 (fp32, each rounded once). */
void or_fp8_quant_row(const float* x, int n, uint8_t* codes, float* scale) {
    float a = 0.0f;
    for (int i = 0; i < n; ++i)
        if (fabsf(x[i]) > a) a = fabsf(x[i]);
    if (!(a >= FLT_MIN)) {
        *scale = 0.0f;
        memset(codes, 0, (size_t)n);
        return;
    }
    const float inv = 448.0f / a;
    *scale = a / 448.0f;
    for (int i = 0; i < n; ++i) codes[i] = or_e4m3_encode(x[i] * inv);
}

/* Byte offsets inside the block of one (layer, page, head), 2*16*D + 128 bytes:
 * K codes [16][D] (16-byte chunks of token t's row rotated by XOR (t & 7)),
 * V codes [D][16] (token order 0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15),
 * 16 K scales, 16 V scales (fp32). */
static inline int64_t or_fp8_k_off(int t, int d, int D) { return (int64_t)t * D + ((((d >> 4) ^ (t & 7))) << 4) + (d & 15); }
static inline int or_fp8_v_pos(int t) { return ((t & 7) >> 1) * 4 + (t & 1) + ((t >> 3) << 1); }
static inline int64_t or_fp8_v_off(int t, int d, int D, int P) { return (int64_t)P * D + (int64_t)d * P + or_fp8_v_pos(t); }
static inline int64_t or_fp8_scale_off(int kv, int t, int D, int P) { return 2LL * P * D + (kv * P + t) * 4; }
static inline int64_t or_fp8_block(int Hkv, int D, int P, int num_pages, int layer, int page, int h) {
    return (((int64_t)layer * num_pages + page) * Hkv + h) * (2LL * P * D + 8LL * P);
}

/*
 * KVCache::append (src/kv_cache.cpp:84-128) into an FP8 pool: token t of
 * sequence b at pos = positions[b] + t, every KV head, K and V rows given in
 * fp32 [B, T, Hkv, D] (fp16 inputs are widened exactly by the caller; a
 * rotated K is rotated before).  Returns 0, or -1 when an entry was skipped.
 */
int or_append_fp8(uint8_t* pool, int L, int Hkv, int D, int P, int num_pages, int layer, const float* k,
                  const float* v, const int32_t* block_tables, int bt_stride, const int32_t* positions, int B,
                  int T) {
    (void)L;
    int bad = 0;
    uint8_t* kc = (uint8_t*)malloc((size_t)D);
    uint8_t* vc = (uint8_t*)malloc((size_t)D);
    for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) {
            const int pos = positions[b] + t;
            if (pos < 0 || pos / P >= bt_stride) {
                bad = 1;
                continue;
            }
            const int32_t page = block_tables[(int64_t)b * bt_stride + pos / P];
            if (page < 0 || page >= num_pages) {
                bad = 1;
                continue;
            }
            const int slot = pos % P;
            for (int h = 0; h < Hkv; ++h) {
                const int64_t src = (((int64_t)b * T + t) * Hkv + h) * D;
                float ks, vs;
                or_fp8_quant_row(k + src, D, kc, &ks);
                or_fp8_quant_row(v + src, D, vc, &vs);
                uint8_t* blk = pool + or_fp8_block(Hkv, D, P, num_pages, layer, page, h);
                for (int d = 0; d < D; ++d) {
                    blk[or_fp8_k_off(slot, d, D)] = kc[d];
                    blk[or_fp8_v_off(slot, d, D, P)] = vc[d];
                }
                memcpy(blk + or_fp8_scale_off(0, slot, D, P), &ks, 4);
                memcpy(blk + or_fp8_scale_off(1, slot, D, P), &vs, 4);
            }
        }
    free(kc);
    free(vc);
    return bad ? -1 : 0;
}

/* Dequantised copy of an FP8 pool: out fp32 [L][num_pages][Hkv][2][P][D],
 * value = code * scale. */
void or_dequant_fp8(const uint8_t* pool, int L, int Hkv, int D, int P, int num_pages, float* out) {
    for (int layer = 0; layer < L; ++layer)
        for (int page = 0; page < num_pages; ++page)
            for (int h = 0; h < Hkv; ++h) {
                const uint8_t* blk = pool + or_fp8_block(Hkv, D, P, num_pages, layer, page, h);
                float* o = out + (((int64_t)layer * num_pages + page) * Hkv + h) * 2LL * P * D;
                for (int t = 0; t < P; ++t) {
                    float ks, vs;
                    memcpy(&ks, blk + or_fp8_scale_off(0, t, D, P), 4);
                    memcpy(&vs, blk + or_fp8_scale_off(1, t, D, P), 4);
                    for (int d = 0; d < D; ++d) {
                        o[(int64_t)t * D + d] = or_e4m3_decode(blk[or_fp8_k_off(t, d, D)]) * ks;
                        o[((int64_t)P + t) * D + d] = or_e4m3_decode(blk[or_fp8_v_off(t, d, D, P)]) * vs;
                    }
                }
            }
}

void or_e4m3_encode_array(const float* x, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = or_e4m3_encode(x[i]);
}

void or_e4m3_decode_array(const uint8_t* c, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = or_e4m3_decode(c[i]);
}

/* launch_matmul's contract (cuda/matmul.cu:42-103): C[M,N] = A[M,K] * B[K,N],
 * all row-major fp32.  matmul_kernel gives each output element to one thread
 * that starts from 0 and adds A[row,k] * B[k,col] for k = 0..K-1 in order (tile
 * by tile, k inside a tile in order); nvcc compiles `sum += a * b` into one
 * fused multiply-add, so this loop uses fmaf in the same order and matches the
 * compiled reference bit for bit. */
void or_matmul(const float* A, const float* B, float* C, int M, int K, int N, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int row = 0; row < M; ++row) {
        for (int col = 0; col < N; ++col) {
            float sum = 0.0f;
            for (int k = 0; k < K; ++k) sum = fmaf(A[(int64_t)row * K + k], B[(int64_t)k * N + col], sum);
            C[(int64_t)row * N + col] = sum;
        }
    }
}
