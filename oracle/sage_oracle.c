/*
 * CPU oracle for the SageAttention2 hot path -- TEST INFRASTRUCTURE ONLY.
 * See sage_oracle.h for what it restates and who may call it.
 *
 * Compiled with -O2 -ffp-contract=off and without -ffast-math: every
 * rounding happens where the C source says, and the FMA contractions that
 * nvcc applies to the reference CUDA source are written out as fmaf().
 */
#include "sage_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ codecs */

static inline float bits_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static inline uint32_t f32_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

/* reference.rs:8-10 */
float or_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* reference.rs:13-20: round to nearest even, NaN stays NaN. */
uint16_t or_f32_to_bf16(float x) {
    uint32_t bits = f32_bits(x);
    if (isnan(x)) return (uint16_t)((bits >> 16) | 0x40);
    uint32_t round = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + round) >> 16);
}

/* reference.rs:23-36: 0x7f / 0xff are NaN. */
float or_e4m3_to_f32(uint8_t b) {
    float sign = (b & 0x80) ? -1.0f : 1.0f;
    int exp = (b >> 3) & 0xf;
    int man = b & 7;
    if (exp == 15 && man == 7) return NAN;
    float mag = exp == 0 ? (float)man * ldexpf(1.0f, -9) : (1.0f + (float)man / 8.0f) * ldexpf(1.0f, exp - 7);
    return sign * mag;
}

/* reference.rs:40-70: round to nearest even, saturate at +-448, NaN -> 0x7f
 * (the semantics of cvt.rn.satfinite.e4m3x2.f32). */
uint8_t or_f32_to_e4m3(float x) {
    if (isnan(x)) return 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0;
    float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7e;
    int e;
    if (a < ldexpf(1.0f, -6)) {
        e = -6;
    } else {
        int ex;
        frexpf(a, &ex); /* a = m * 2^ex, m in [0.5, 1) */
        e = ex - 1;
    }
    double step = ldexp(1.0, e - 3);
    unsigned k = (unsigned)nearbyint((double)a / step);
    if (k == 16) {
        e += 1;
        k = 8;
    }
    if (e == -6 && k < 8) return sign | (uint8_t)k;
    if (e > 8 || (e == 8 && k > 14)) return sign | 0x7e;
    return sign | (uint8_t)((e + 7) << 3) | (uint8_t)(k - 8);
}

void or_f32_to_e4m3_n(const float* x, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = or_f32_to_e4m3(x[i]);
}

/* reference.rs:74-76 / sage_common.cu:155 */
int or_vpos(int k) { return ((k >> 1) & 3) * 4 + ((k >> 3) << 1) + (k & 1); }

/* __float2int_rn then clamp to [-127, 127] (sage_common.cu:95-99). */
static inline int8_t s8(float x) {
    if (isnan(x)) return -127;
    float r = nearbyintf(x);
    if (r > 127.0f) r = 127.0f;
    if (r < -127.0f) r = -127.0f;
    return (int8_t)(int)r;
}

/* ------------------------------------------------------------------ RNG */

/* reference.rs:235-241 */
uint64_t or_rng_next(uint64_t* s) {
    *s += 0x9e3779b97f4a7c15ull;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* reference.rs:244-246 */
double or_rng_uniform(uint64_t* s) { return (double)(or_rng_next(s) >> 11) / (double)(1ull << 53); }

/* reference.rs:249-253 */
float or_rng_normal(uint64_t* s) {
    double u1 = or_rng_uniform(s);
    if (u1 < 1e-300) u1 = 1e-300;
    double u2 = or_rng_uniform(s);
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

void or_rng_normals(uint64_t* s, float* out, int64_t n, float std_, float mean) {
    for (int64_t i = 0; i < n; i++) out[i] = or_rng_normal(s) * std_ + mean;
}

/* platform/spl-nn/src/sage/tests.rs:300-329 */
void or_synthetic(int batch, int heads, int tokens, int d, uint64_t seed, uint16_t* q, uint16_t* k,
                  uint16_t* v) {
    uint64_t s = seed;
    const int clusters = 37;
    float* centers = (float*)malloc(sizeof(float) * (size_t)clusters * heads * d);
    float* k_off = (float*)malloc(sizeof(float) * (size_t)heads * d);
    float* v_off = (float*)malloc(sizeof(float) * (size_t)heads * d);
    for (int64_t i = 0; i < (int64_t)clusters * heads * d; i++) centers[i] = or_rng_normal(&s);
    for (int i = 0; i < heads * d; i++) k_off[i] = 3.0f * or_rng_normal(&s);
    for (int i = 0; i < heads * d; i++) v_off[i] = 2.0f * or_rng_normal(&s);
    for (int b = 0; b < batch; b++)
        for (int t = 0; t < tokens; t++) {
            int c = (int)(or_rng_next(&s) % (uint64_t)clusters);
            for (int h = 0; h < heads; h++)
                for (int x = 0; x < d; x++) {
                    int64_t i = (((int64_t)b * tokens + t) * heads + h) * d + x;
                    float ctr = centers[((int64_t)c * heads + h) * d + x];
                    float outlier = (x % 23 == 5) ? 6.0f : 1.0f;
                    float qv = 1.6f * ctr + 0.6f * or_rng_normal(&s);
                    float kv = (1.6f * ctr + 0.6f * or_rng_normal(&s)) * outlier + k_off[h * d + x];
                    float vv = or_rng_normal(&s) + 0.5f * ctr + v_off[h * d + x];
                    q[i] = or_f32_to_bf16(qv);
                    k[i] = or_f32_to_bf16(kv);
                    v[i] = or_f32_to_bf16(vv);
                }
        }
    free(centers);
    free(k_off);
    free(v_off);
}

/* ------------------------------------------------------------------ merge geometry */

/* sage_quant.cu:210-235 */
int or_members(const or_geom* g, int j, int* base, int* nx) {
    if (g->merge == 1) {
        *base = j;
        *nx = 1;
        return 1;
    }
    int dense = g->dense_frames * g->frame_tokens;
    if (j < dense) {
        *base = j;
        *nx = 1;
        return 1;
    }
    int f = g->dense_frames + (j - dense) / g->merged_frame, loc = (j - dense) % g->merged_frame;
    if (loc < g->special) {
        *base = f * g->frame_tokens + loc;
        *nx = 1;
        return 1;
    }
    int cell = loc - g->special;
    int gy = cell / g->merged_w, gx = cell % g->merged_w;
    int y0 = gy * g->merge, x0 = gx * g->merge;
    int ny = g->merge < g->grid_h - y0 ? g->merge : g->grid_h - y0;
    int n = g->merge < g->grid_w - x0 ? g->merge : g->grid_w - x0;
    *nx = n;
    *base = f * g->frame_tokens + g->special + y0 * g->grid_w + x0;
    return ny * n;
}

/* ------------------------------------------------------------------ quantiser */

/* The device LayerNorm of sage_quant.cu:34-52 over one head row, with the
 * same summation tree (8 channels per lane, xor butterfly over D/8 lanes)
 * and 1/sqrtf in place of rsqrtf.  Out of the bit gate (rsqrtf is not
 * reproducible), tolerance-checked only. */
static void dev_layernorm(float* x, const float* w, const float* bias, int d, float eps) {
    int ch = d / 8;
    float part[16] = {0.f}, part2[16] = {0.f};  /* d is 64 or 128: ch = 8 or 16 lanes */
    for (int c = 0; c < ch; c++) {
        float s = 0.f;
        for (int e = 0; e < 8; e++) s += x[c * 8 + e];
        part[c] = s;
    }
    for (int o = 1; o < ch; o <<= 1) {
        float nxt[16];
        for (int c = 0; c < ch; c++) nxt[c] = part[c] + part[c ^ o];
        memcpy(part, nxt, sizeof(float) * ch);
    }
    float mean = part[0] * (1.0f / (float)d);
    for (int c = 0; c < ch; c++) {
        float s2 = 0.f;
        for (int e = 0; e < 8; e++) {
            float t = x[c * 8 + e] - mean;
            s2 = fmaf(t, t, s2);
        }
        part2[c] = s2;
    }
    for (int o = 1; o < ch; o <<= 1) {
        float nxt[16];
        for (int c = 0; c < ch; c++) nxt[c] = part2[c] + part2[c ^ o];
        memcpy(part2, nxt, sizeof(float) * ch);
    }
    float rstd = 1.0f / sqrtf(fmaf(part2[0], 1.0f / (float)d, eps));
    for (int i = 0; i < d; i++) x[i] = fmaf((x[i] - mean) * rstd, w[i], bias[i]);
}

static inline void load_row(const uint16_t* p, int d, float* out) {
    for (int i = 0; i < d; i++) out[i] = or_bf16_to_f32(p[i]);
}

/* sg_prep, Q role (sage_quant.cu:84-127) for one (tile, q head, batch). */
static void prep_q(const uint16_t* q, const float* ln, int8_t* q8, float* q_scale, const or_geom* g, int tile,
                   int h, int b) {
    const int d = g->d;
    float* rows = (float*)malloc(sizeof(float) * OR_QTILE * d);
    float gmax[OR_QTILE / OR_QGROUP];
    for (int i = 0; i < OR_QTILE / OR_QGROUP; i++) gmax[i] = 0.f;
    for (int tl = 0; tl < OR_QTILE; tl++) {
        int tok = tile * OR_QTILE + tl;
        float* f = rows + (int64_t)tl * d;
        if (tok < g->tokens) {
            load_row(q + (int64_t)b * g->q_sb + (int64_t)tok * g->q_st + (int64_t)h * g->q_sh, d, f);
            if (g->flags & OR_LN_Q) dev_layernorm(f, ln, ln + d, d, g->ln_eps);
        } else {
            for (int i = 0; i < d; i++) f[i] = 0.f;
        }
        for (int i = 0; i < d; i++) {
            float a = fabsf(f[i]);
            if (a > gmax[tl / OR_QGROUP]) gmax[tl / OR_QGROUP] = a;
        }
    }
    const int64_t bh = (int64_t)b * g->heads + h;
    for (int tl = 0; tl < OR_QTILE; tl++) {
        float amax = gmax[tl / OR_QGROUP];
        float inv = amax > 0.f ? 127.0f / amax : 0.f;
        int8_t* dst = q8 + (bh * g->tq_pad + (int64_t)tile * OR_QTILE + tl) * d;
        for (int i = 0; i < d; i++) dst[i] = s8(rows[(int64_t)tl * d + i] * inv);
    }
    for (int gi = 0; gi < OR_QTILE / OR_QGROUP; gi++) {
        float t = gmax[gi] * (1.0f / 127.0f);
        q_scale[bh * (g->tq_pad / OR_QGROUP) + (int64_t)tile * (OR_QTILE / OR_QGROUP) + gi] = t * g->q_mul;
    }
    free(rows);
}

/* sg_prep, statistics role (sage_quant.cu:73-107, 129-159) for one
 * (tile, kv head, batch): the per-thread sequential sums, the xor butterfly
 * over lanes CH..16 and the sequential sum over the 8 warps. */
static void prep_stats(const uint16_t* k, const uint16_t* v, const float* ln, float* part, const or_geom* g,
                       int tile, int h, int b) {
    const int d = g->d, CH = d / 8, TPI = 256 / CH, NI = OR_QTILE / TPI;
    /* acc[stat][tid][e] */
    float(*acc)[256][8] = (float(*)[256][8])malloc(sizeof(float) * 4 * 256 * 8);
    float fk[128], fv[128];
    for (int tid = 0; tid < 256; tid++) {
        int ch = tid % CH;
        for (int e = 0; e < 8; e++) {
            acc[0][tid][e] = 0.f;
            acc[1][tid][e] = 0.f;
            acc[2][tid][e] = 3.0e38f;
            acc[3][tid][e] = -3.0e38f;
        }
        for (int i = 0; i < NI; i++) {
            int tl = tid / CH + i * TPI;
            int tok = tile * OR_QTILE + tl;
            if (tok >= g->tokens) continue;
            load_row(k + (int64_t)b * g->k_sb + (int64_t)tok * g->k_st + (int64_t)h * g->k_sh, d, fk);
            load_row(v + (int64_t)b * g->v_sb + (int64_t)tok * g->v_st + (int64_t)h * g->v_sh, d, fv);
            if (g->flags & OR_LN_K) dev_layernorm(fk, ln + 2 * d, ln + 3 * d, d, g->ln_eps);
            for (int e = 0; e < 8; e++) {
                float kk = fk[ch * 8 + e], vv = fv[ch * 8 + e];
                acc[0][tid][e] += kk;
                acc[1][tid][e] += vv;
                acc[2][tid][e] = fminf(acc[2][tid][e], vv);
                acc[3][tid][e] = fmaxf(acc[3][tid][e], vv);
            }
        }
    }
    /* xor butterfly inside each warp, offsets CH, 2CH, ..., 16 */
    for (int w = 0; w < 8; w++)
        for (int o = CH; o < 32; o <<= 1) {
            float nxt[4][32][8];
            for (int l = 0; l < 32; l++)
                for (int e = 0; e < 8; e++) {
                    int a = w * 32 + l, p = w * 32 + (l ^ o);
                    nxt[0][l][e] = acc[0][a][e] + acc[0][p][e];
                    nxt[1][l][e] = acc[1][a][e] + acc[1][p][e];
                    nxt[2][l][e] = fminf(acc[2][a][e], acc[2][p][e]);
                    nxt[3][l][e] = fmaxf(acc[3][a][e], acc[3][p][e]);
                }
            for (int s = 0; s < 4; s++)
                for (int l = 0; l < 32; l++)
                    for (int e = 0; e < 8; e++) acc[s][w * 32 + l][e] = nxt[s][l][e];
        }
    /* red[w][stat][ch*8+e] = lane ch of warp w; then r = red[0] (+) red[1..7] */
    const int64_t bh = (int64_t)b * g->kv_heads + h;
    for (int s = 0; s < 4; s++)
        for (int dd = 0; dd < d; dd++) {
            int ch = dd / 8, e = dd % 8;
            float r = acc[s][ch][e];
            for (int w = 1; w < 8; w++) {
                float x = acc[s][w * 32 + ch][e];
                r = s < 2 ? r + x : (s == 2 ? fminf(r, x) : fmaxf(r, x));
            }
            part[((bh * g->q_tiles + tile) * 4 + s) * d + dd] = r;
        }
    free(acc);
}

void or_prep(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* ln, int8_t* q8,
             float* q_scale, float* part, const or_geom* g) {
    for (int b = 0; b < g->batch; b++) {
        for (int h = 0; h < g->heads; h++)
            for (int t = 0; t < g->q_tiles; t++) prep_q(q, ln, q8, q_scale, g, t, h, b);
        for (int h = 0; h < g->kv_heads; h++)
            for (int t = 0; t < g->q_tiles; t++) prep_stats(k, v, ln, part, g, t, h, b);
    }
}

/* sage_quant.cu:163-206 */
void or_finalize(const float* part, float* stats, const or_geom* g) {
    const int d = g->d;
    for (int b = 0; b < g->batch; b++)
        for (int h = 0; h < g->kv_heads; h++) {
            const int64_t bh = (int64_t)b * g->kv_heads + h;
            float st[4][128];
            for (int s = 0; s < 4; s++)
                for (int dd = 0; dd < d; dd++) {
                    const float* p = part + bh * g->q_tiles * 4 * d + s * d + dd;
                    float r0 = s < 2 ? 0.f : (s == 2 ? 3.0e38f : -3.0e38f);
                    float r1 = r0;
                    int t = 0;
                    for (; t + 1 < g->q_tiles; t += 2) {
                        float x0 = p[(int64_t)t * 4 * d], x1 = p[(int64_t)(t + 1) * 4 * d];
                        if (s < 2) {
                            r0 += x0;
                            r1 += x1;
                        } else if (s == 2) {
                            r0 = fminf(r0, x0);
                            r1 = fminf(r1, x1);
                        } else {
                            r0 = fmaxf(r0, x0);
                            r1 = fmaxf(r1, x1);
                        }
                    }
                    if (t < g->q_tiles) {
                        float x0 = p[(int64_t)t * 4 * d];
                        r0 = s < 2 ? r0 + x0 : (s == 2 ? fminf(r0, x0) : fmaxf(r0, x0));
                    }
                    st[s][dd] = s < 2 ? r0 + r1 : (s == 2 ? fminf(r0, r1) : fmaxf(r0, r1));
                }
            for (int dd = 0; dd < d; dd++) {
                float n = (float)g->tokens;
                float mk = (g->flags & OR_SMOOTH_K) ? st[0][dd] / n : 0.f;
                float mv = (g->flags & OR_SMOOTH_V) ? st[1][dd] / n : 0.f;
                float amax = fmaxf(st[3][dd] - mv, mv - st[2][dd]);
                float scale = amax > 0.f ? amax / g->v_range : 1.0f;
                float* o = stats + bh * 4 * d;
                o[dd] = mk;
                o[d + dd] = mv;
                o[2 * d + dd] = scale;
                o[3 * d + dd] = 1.0f / scale;
            }
        }
}

/* sage_quant.cu:238-326 */
void or_quant_kv(const uint16_t* k, const uint16_t* v, const float* ln, const float* stats, int8_t* k8,
                 float* k_scale, uint8_t* v8, float* kbias, const or_geom* g) {
    const int d = g->d, nblk = g->tk_pad / OR_KBLOCK;
    float* kv = (float*)malloc(sizeof(float) * OR_KBLOCK * d);
    float fk[128], fv[128], ksum[128], vsum[128];
    for (int b = 0; b < g->batch; b++)
        for (int h = 0; h < g->kv_heads; h++) {
            const int64_t bh = (int64_t)b * g->kv_heads + h;
            const float* st = stats + bh * 4 * d;
            for (int blk = 0; blk < nblk; blk++) {
                float amax = 0.f;
                uint8_t* vo = v8 + (bh * nblk + blk) * (int64_t)(d * OR_KBLOCK);
                for (int kl = 0; kl < OR_KBLOCK; kl++) {
                    int j = blk * OR_KBLOCK + kl;
                    int ok = j < g->tk;
                    int base = 0, nx = 1;
                    int cnt = ok ? or_members(g, j, &base, &nx) : 0;
                    for (int i = 0; i < d; i++) ksum[i] = vsum[i] = 0.f;
                    for (int m = 0; m < cnt; m++) {
                        int tok = base + (m / nx) * g->grid_w + m % nx;
                        load_row(k + (int64_t)b * g->k_sb + (int64_t)tok * g->k_st + (int64_t)h * g->k_sh, d, fk);
                        load_row(v + (int64_t)b * g->v_sb + (int64_t)tok * g->v_st + (int64_t)h * g->v_sh, d, fv);
                        if (g->flags & OR_LN_K) dev_layernorm(fk, ln + 2 * d, ln + 3 * d, d, g->ln_eps);
                        for (int i = 0; i < d; i++) {
                            ksum[i] += fk[i];
                            vsum[i] += fv[i];
                        }
                    }
                    float rc = cnt > 0 ? 1.0f / (float)cnt : 0.f;
                    int col = (kl & ~15) + or_vpos(kl & 15);
                    for (int i = 0; i < d; i++) {
                        /* nvcc contracts `ksum * rc - mean` and `vsum * rc - mv` to FFMA */
                        float x = ok ? fmaf(ksum[i], rc, -st[i]) : 0.f;
                        kv[kl * d + i] = x;
                        if (fabsf(x) > amax) amax = fabsf(x);
                        float vq = ok ? fmaf(vsum[i], rc, -st[d + i]) * st[3 * d + i] : 0.f;
                        vo[i * OR_KBLOCK + col] = or_f32_to_e4m3(vq);
                    }
                }
                float inv = amax > 0.f ? 127.0f / amax : 0.f;
                for (int kl = 0; kl < OR_KBLOCK; kl++) {
                    int8_t* dst = k8 + (bh * g->tk_pad + (int64_t)blk * OR_KBLOCK + kl) * d;
                    for (int i = 0; i < d; i++) dst[i] = s8(kv[kl * d + i] * inv);
                }
                k_scale[bh * nblk + blk] = amax * (1.0f / 127.0f);
                if (g->merge > 1 && b == 0 && h == 0 && kbias) {
                    for (int t = 0; t < OR_KBLOCK; t++) {
                        int j = blk * OR_KBLOCK + t, base, nx;
                        kbias[j] = j < g->tk ? log2f((float)or_members(g, j, &base, &nx)) : -INFINITY;
                    }
                }
            }
        }
    free(kv);
}

void or_prepare(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* ln, int8_t* q8,
                float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8, float* stats, float* kbias,
                float* part, const or_geom* g) {
    or_prep(q, k, v, ln, q8, q_scale, part, g);
    or_finalize(part, stats, g);
    or_quant_kv(k, v, ln, stats, k8, k_scale, v8, kbias, g);
}

/* ------------------------------------------------------------------ attention */

/* reference.rs:110-118 */
void or_layer_norm(float* x, const float* w, const float* b, int n, float eps) {
    double mean = 0.0, var = 0.0;
    for (int i = 0; i < n; i++) mean += (double)x[i];
    mean /= n;
    for (int i = 0; i < n; i++) var += ((double)x[i] - mean) * ((double)x[i] - mean);
    var /= n;
    double rstd = 1.0 / sqrt(var + (double)eps);
    for (int i = 0; i < n; i++) x[i] = (float)(((double)x[i] - mean) * rstd * (double)w[i] + (double)b[i]);
}

/* reference.rs:148-184, plus an optional causal mask (an extension). */
void or_attention_f64(const float* q, const float* k, const float* v, const float* bias_log2, int tq, int tk,
                      int d, float scale, int causal, int causal_offset, float* out) {
    double* logits = (double*)malloc(sizeof(double) * (size_t)tk);
    double* acc = (double*)malloc(sizeof(double) * (size_t)d);
    for (int i = 0; i < tq; i++) {
        const float* qi = q + (int64_t)i * d;
        int nk = tk;
        if (causal) {
            nk = i + causal_offset + 1;
            if (nk > tk) nk = tk;
            if (nk < 0) nk = 0;
        }
        double mx = -INFINITY;
        for (int j = 0; j < nk; j++) {
            const float* kj = k + (int64_t)j * d;
            double dot = 0.0;
            for (int c = 0; c < d; c++) dot += (double)qi[c] * (double)kj[c];
            logits[j] = dot * (double)scale + (bias_log2 ? (double)bias_log2[j] * 0.6931471805599453 : 0.0);
            if (logits[j] > mx) mx = logits[j];
        }
        double sum = 0.0;
        for (int c = 0; c < d; c++) acc[c] = 0.0;
        for (int j = 0; j < nk; j++) {
            double p = exp(logits[j] - mx);
            sum += p;
            const float* vj = v + (int64_t)j * d;
            for (int c = 0; c < d; c++) acc[c] += p * (double)vj[c];
        }
        for (int c = 0; c < d; c++) out[(int64_t)i * d + c] = (float)(acc[c] / sum);
    }
    free(logits);
    free(acc);
}

/* ---- threaded whole-tensor f64 attention ---- */

typedef struct {
    const uint16_t *q, *k, *v;
    const or_geom* g;
    float scale;
    int causal, row0, row1;
    float* out;
    /* merged K/V per (b, kv head): [b][hkv][tk][d] f32 and kbias [tk] */
    const float *km, *vm, *bias;
    int64_t next; /* work counter */
    pthread_mutex_t mu;
} att_job;

static void* att_worker(void* arg) {
    att_job* J = (att_job*)arg;
    const or_geom* g = J->g;
    const int d = g->d, group = g->heads / g->kv_heads, rows = J->row1 - J->row0;
    const int chunk = 16;
    const int per_bh = (rows + chunk - 1) / chunk;
    const int64_t total = (int64_t)g->batch * g->heads * per_bh;
    float* qrow = (float*)malloc(sizeof(float) * (size_t)chunk * d);
    float* orow = (float*)malloc(sizeof(float) * (size_t)chunk * d);
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t w = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (w >= total) break;
        int c = (int)(w % per_bh);
        int64_t bh = w / per_bh;
        int h = (int)(bh % g->heads), b = (int)(bh / g->heads);
        int r0 = J->row0 + c * chunk, r1 = r0 + chunk;
        if (r1 > J->row1) r1 = J->row1;
        for (int r = r0; r < r1; r++)
            load_row(J->q + (int64_t)b * g->q_sb + (int64_t)r * g->q_st + (int64_t)h * g->q_sh, d,
                     qrow + (int64_t)(r - r0) * d);
        const int64_t kvh = (int64_t)b * g->kv_heads + h / group;
        const float* kb = J->km + kvh * (int64_t)g->tk * d;
        const float* vb = J->vm + kvh * (int64_t)g->tk * d;
        or_attention_f64(qrow, kb, vb, J->bias, r1 - r0, g->tk, d, J->scale, J->causal, r0, orow);
        for (int r = r0; r < r1; r++)
            memcpy(J->out + (((int64_t)b * g->tokens + r) * g->heads + h) * d, orow + (int64_t)(r - r0) * d,
                   sizeof(float) * d);
    }
    free(qrow);
    free(orow);
    return NULL;
}

int or_attention_bthd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const or_geom* g, float scale,
                      int causal, int row0, int row1, int nthreads, float* out) {
    const int d = g->d;
    /* merged (or plain) K and V per (b, kv head), as reference.rs:123-143 */
    float* km = (float*)calloc((size_t)g->batch * g->kv_heads * g->tk * d, sizeof(float));
    float* vm = (float*)calloc((size_t)g->batch * g->kv_heads * g->tk * d, sizeof(float));
    float* bias = g->merge > 1 ? (float*)malloc(sizeof(float) * (size_t)g->tk) : NULL;
    float* fk = (float*)malloc(sizeof(float) * d);
    float* fv = (float*)malloc(sizeof(float) * d);
    for (int b = 0; b < g->batch; b++)
        for (int h = 0; h < g->kv_heads; h++) {
            float* kb = km + ((int64_t)b * g->kv_heads + h) * (int64_t)g->tk * d;
            float* vb = vm + ((int64_t)b * g->kv_heads + h) * (int64_t)g->tk * d;
            for (int j = 0; j < g->tk; j++) {
                int base, nx, cnt = or_members(g, j, &base, &nx);
                for (int m = 0; m < cnt; m++) {
                    int tok = base + (m / nx) * g->grid_w + m % nx;
                    load_row(k + (int64_t)b * g->k_sb + (int64_t)tok * g->k_st + (int64_t)h * g->k_sh, d, fk);
                    load_row(v + (int64_t)b * g->v_sb + (int64_t)tok * g->v_st + (int64_t)h * g->v_sh, d, fv);
                    for (int c = 0; c < d; c++) {
                        kb[(int64_t)j * d + c] += fk[c];
                        vb[(int64_t)j * d + c] += fv[c];
                    }
                }
                float n = (float)cnt;
                for (int c = 0; c < d; c++) {
                    kb[(int64_t)j * d + c] /= n;
                    vb[(int64_t)j * d + c] /= n;
                }
                if (bias) bias[j] = log2f(n);
            }
        }
    free(fk);
    free(fv);
    att_job J;
    J.q = q;
    J.k = k;
    J.v = v;
    J.g = g;
    J.scale = scale;
    J.causal = causal;
    J.row0 = row0;
    J.row1 = row1;
    J.out = out;
    J.km = km;
    J.vm = vm;
    J.bias = bias;
    J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, att_worker, &J);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&J.mu);
    free(km);
    free(vm);
    free(bias);
    return 0;
}

/* ---- emulation of the quantised kernel's arithmetic ---- */

typedef struct {
    const int8_t* q8;
    const float* q_scale;
    const int8_t* k8;
    const float* k_scale;
    const uint8_t* v8;
    const float* stats;
    const float* kbias;
    const or_geom* g;
    int causal;
    int row0, row1;
    float* out;
    int64_t next;
    pthread_mutex_t mu;
} emu_job;

static void* emu_worker(void* arg) {
    emu_job* J = (emu_job*)arg;
    const or_geom* g = J->g;
    const int d = g->d, group = g->heads / g->kv_heads, nkb = g->tk_pad / OR_KBLOCK;
    double* x = (double*)malloc(sizeof(double) * (size_t)g->tk);
    double* acc = (double*)malloc(sizeof(double) * d);
    float* vdq = (float*)malloc(sizeof(float) * (size_t)g->tk * d);
    int64_t cur_kvh = -1;
    const int64_t total = (int64_t)g->batch * g->heads;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t w = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (w >= total) break;
        int h = (int)(w % g->heads), b = (int)(w / g->heads);
        int64_t bh = (int64_t)b * g->heads + h, kvh = (int64_t)b * g->kv_heads + h / group;
        if (kvh != cur_kvh) {
            for (int j = 0; j < g->tk; j++) {
                int blk = j / OR_KBLOCK, kl = j % OR_KBLOCK, col = (kl & ~15) + or_vpos(kl & 15);
                for (int c = 0; c < d; c++)
                    vdq[(int64_t)j * d + c] =
                        or_e4m3_to_f32(J->v8[((kvh * nkb + blk) * d + c) * (int64_t)OR_KBLOCK + col]);
            }
            cur_kvh = kvh;
        }
        const float* st = J->stats + kvh * 4 * d;
        for (int i = J->row0; i < J->row1; i++) {
            const int8_t* qi = J->q8 + (bh * g->tq_pad + i) * d;
            double qs = J->q_scale[bh * (g->tq_pad / OR_QGROUP) + i / OR_QGROUP];
            int nk = J->causal ? (i + 1 < g->tk ? i + 1 : g->tk) : g->tk;
            double mx = -INFINITY;
            for (int j = 0; j < nk; j++) {
                const int8_t* kj = J->k8 + (kvh * g->tk_pad + j) * d;
                int32_t s = 0;
                for (int c = 0; c < d; c++) s += (int32_t)qi[c] * (int32_t)kj[c];
                x[j] = (double)s * qs * (double)J->k_scale[kvh * nkb + j / OR_KBLOCK] +
                       (J->kbias && g->merge > 1 ? (double)J->kbias[j] : 0.0);
                if (x[j] > mx) mx = x[j];
            }
            double l = 0.0;
            for (int c = 0; c < d; c++) acc[c] = 0.0;
            for (int j = 0; j < nk; j++) {
                double p = 448.0 * exp2(x[j] - mx);
                l += p;
                double p8 = (double)or_e4m3_to_f32(or_f32_to_e4m3((float)p));
                for (int c = 0; c < d; c++) acc[c] += p8 * (double)vdq[(int64_t)j * d + c];
            }
            float* o = J->out + (((int64_t)b * g->tokens + i) * g->heads + h) * d;
            for (int c = 0; c < d; c++) o[c] = (float)(acc[c] / l * (double)st[2 * d + c] + (double)st[d + c]);
        }
    }
    free(x);
    free(acc);
    free(vdq);
    return NULL;
}

void or_sage_emulate(const int8_t* q8, const float* q_scale, const int8_t* k8, const float* k_scale,
                     const uint8_t* v8, const float* stats, const float* kbias, const or_geom* g, int causal,
                     int row0, int row1, int nthreads, float* out) {
    emu_job J;
    J.q8 = q8;
    J.q_scale = q_scale;
    J.k8 = k8;
    J.k_scale = k_scale;
    J.v8 = v8;
    J.stats = stats;
    J.kbias = kbias;
    J.g = g;
    J.causal = causal;
    J.row0 = row0 < 0 ? 0 : row0;
    J.row1 = row1 > g->tokens ? g->tokens : row1;
    J.out = out;
    J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, emu_worker, &J);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&J.mu);
}

/* ---- online-softmax emulation (the kernels' block-by-block arithmetic) ---- */

/* The reference kernel's online softmax (platform/spl-nn/cuda/sage_attn.cu:
 * 227-344, SG_FAST_EXP): keys in blocks; S read as the float 1.5 * 2^23 + S;
 * per block m_new = max(m, max_key fmaf(x, sc, -M * sc)) with sc = q_scale *
 * k_scale of the key's 64-key group (merged: x = fmaf(x, sc, bias - M * sc)
 * is the log2 logit, m_new = max(m, max x)); alpha = 2^(m - m_new);
 * p = 2^(fmaf(x, sc, (log2 448 - m_new) + (-M * sc))); l = fmaf(l, alpha,
 * sum p); the block's P8 V8 summed from zero and folded O = fmaf(O, alpha,
 * PV); out = fmaf(O * (1 / l), v_scale, v_mean) (:405-420).  `block` = 64 is
 * the reference kernel's block; 128 is this library's (one max per 128 keys,
 * two k_scale groups).  Extensions: causal keys j <= i, GQA.  exp2 is the C
 * library's (the kernels use ex2.approx), and each block's PV is summed in
 * double and rounded once (the tensor cores sum in FP32), so the emulation
 * agrees with a kernel to rounding noise, not bit for bit. */
typedef struct {
    const int8_t* q8;
    const float* q_scale;
    const int8_t* k8;
    const float* k_scale;
    const uint8_t* v8;
    const float* stats;
    const float* kbias;
    const or_geom* g;
    int causal, block, row0, row1;
    float* out;
    int64_t next;
    pthread_mutex_t mu;
} onl_job;

static void* onl_worker(void* arg) {
    onl_job* J = (onl_job*)arg;
    const or_geom* g = J->g;
    const int d = g->d, group = g->heads / g->kv_heads, nkb = g->tk_pad / OR_KBLOCK, B = J->block;
    const int merge = J->kbias && g->merge > 1;
    const float M = 12582912.0f, L448 = 8.807354922057604f;
    float* vdq = (float*)malloc(sizeof(float) * (size_t)g->tk_pad * d);
    float* xf = (float*)malloc(sizeof(float) * (size_t)B);
    double* c = (double*)malloc(sizeof(double) * d);
    float* o = (float*)malloc(sizeof(float) * d);
    int64_t cur_kvh = -1;
    const int64_t total = (int64_t)g->batch * g->heads;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t w = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (w >= total) break;
        int h = (int)(w % g->heads), b = (int)(w / g->heads);
        int64_t bh = (int64_t)b * g->heads + h, kvh = (int64_t)b * g->kv_heads + h / group;
        if (kvh != cur_kvh) {
            for (int j = 0; j < g->tk_pad; j++) {
                int blk = j / OR_KBLOCK, kl = j % OR_KBLOCK, col = (kl & ~15) + or_vpos(kl & 15);
                for (int ch = 0; ch < d; ch++)
                    vdq[(int64_t)j * d + ch] =
                        or_e4m3_to_f32(J->v8[((kvh * nkb + blk) * d + ch) * (int64_t)OR_KBLOCK + col]);
            }
            cur_kvh = kvh;
        }
        const float* st = J->stats + kvh * 4 * d;
        for (int i = J->row0; i < J->row1; i++) {
            const int8_t* qi = J->q8 + (bh * g->tq_pad + i) * d;
            const float qs = J->q_scale[bh * (g->tq_pad / OR_QGROUP) + i / OR_QGROUP];
            const int nk = J->causal ? (i + 1 < g->tk ? i + 1 : g->tk) : g->tk;
            float m = -INFINITY, l = 0.f;
            for (int ch = 0; ch < d; ch++) o[ch] = 0.f;
            for (int k0 = 0; k0 < nk; k0 += B) {
                float mnew = m;
                for (int t = 0; t < B; t++) {
                    const int j = k0 + t;
                    if (j >= nk) {
                        xf[t] = -INFINITY;
                        continue;
                    }
                    const int8_t* kj = J->k8 + (kvh * g->tk_pad + j) * d;
                    int32_t sacc = 0;
                    for (int ch = 0; ch < d; ch++) sacc += (int32_t)qi[ch] * (int32_t)kj[ch];
                    const float sc = qs * J->k_scale[kvh * nkb + j / OR_KBLOCK];
                    const float xm = M + (float)sacc; /* exact: |S| < 2^22 */
                    const float lg = merge ? fmaf(xm, sc, J->kbias[j] - M * sc) : fmaf(xm, sc, -(M * sc));
                    xf[t] = merge ? lg : xm;
                    if (lg > mnew) mnew = lg;
                }
                const float alpha = exp2f(m - mnew);
                m = mnew;
                float sum = 0.f;
                for (int ch = 0; ch < d; ch++) c[ch] = 0.0;
                for (int t = 0; t < B; t++) {
                    const int j = k0 + t;
                    if (j >= nk) continue;
                    float p;
                    if (merge) {
                        p = exp2f(xf[t] + (L448 - mnew));
                    } else {
                        const float sc = qs * J->k_scale[kvh * nkb + j / OR_KBLOCK];
                        p = exp2f(fmaf(xf[t], sc, (L448 - mnew) + (-(M * sc))));
                    }
                    sum += p;
                    const double p8 = (double)or_e4m3_to_f32(or_f32_to_e4m3(p));
                    if (p8 != 0.0)
                        for (int ch = 0; ch < d; ch++) c[ch] += p8 * (double)vdq[(int64_t)j * d + ch];
                }
                l = fmaf(l, alpha, sum);
                for (int ch = 0; ch < d; ch++) o[ch] = fmaf(o[ch], alpha, (float)c[ch]);
            }
            const float inv = 1.0f / l;
            float* out = J->out + (((int64_t)b * g->tokens + i) * g->heads + h) * d;
            for (int ch = 0; ch < d; ch++) out[ch] = fmaf(o[ch] * inv, st[2 * d + ch], st[d + ch]);
        }
    }
    free(vdq);
    free(xf);
    free(c);
    free(o);
    return NULL;
}

void or_sage_online(const int8_t* q8, const float* q_scale, const int8_t* k8, const float* k_scale,
                    const uint8_t* v8, const float* stats, const float* kbias, const or_geom* g, int causal,
                    int block, int row0, int row1, int nthreads, float* out) {
    onl_job J;
    J.q8 = q8;
    J.q_scale = q_scale;
    J.k8 = k8;
    J.k_scale = k_scale;
    J.v8 = v8;
    J.stats = stats;
    J.kbias = kbias;
    J.g = g;
    J.causal = causal;
    J.block = block;
    J.row0 = row0 < 0 ? 0 : row0;
    J.row1 = row1 > g->tokens ? g->tokens : row1;
    J.out = out;
    J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, onl_worker, &J);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&J.mu);
}

/* ------------------------------------------------------------------ metrics */

/* reference.rs:201-225 */
void or_errors(const float* ours, const float* ref, int64_t n, double* out) {
    double dot = 0, na = 0, nr = 0, l1 = 0, l1r = 0, l2 = 0, mx = 0, rmax = 0;
    for (int64_t i = 0; i < n; i++) {
        double a = ours[i], r = ref[i];
        dot += a * r;
        na += a * a;
        nr += r * r;
        l1 += fabs(a - r);
        l1r += fabs(r);
        l2 += (a - r) * (a - r);
        if (fabs(a - r) > mx) mx = fabs(a - r);
        if (fabs(r) > rmax) rmax = fabs(r);
    }
    double den = sqrt(na) * sqrt(nr);
    out[0] = dot / (den > 1e-300 ? den : 1e-300);
    out[1] = l1 / (l1r > 1e-300 ? l1r : 1e-300);
    out[2] = sqrt(l2 / (nr > 1e-300 ? nr : 1e-300));
    out[3] = mx;
    out[4] = rmax;
}

/* mod.rs:905-910 */
double or_flops(int batch, int heads, int tq, int tk, int d) {
    return 4.0 * (double)batch * heads * (double)tq * (double)tk * (double)d;
}

/* ------------------------------------------------------------------ QKV path */

typedef struct {
    const uint16_t *x, *w, *bias;
    const float* rope;
    int rope_half, frame_len, m, n, k, tokens, hq, hkv, d;
    float *q, *kk, *v;
    int64_t next;
    pthread_mutex_t mu;
    /* FP8 variant (x8 != NULL): E4M3 operands and their scales */
    const uint8_t *x8, *w8;
    const float *x_scale, *w_scale;
} qkv_job;

static void* qkv_worker(void* arg) {
    qkv_job* J = (qkv_job*)arg;
    double* y = (double*)malloc(sizeof(double) * (size_t)J->n);
    double* xr = (double*)malloc(sizeof(double) * (size_t)J->k);
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t r = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (r >= J->m) break;
        if (J->x8) {
            /* gemm.rs:294-337 (deferred scales) then qkv.rs:306-330: the
             * products of the E4M3 values, times the token and channel
             * scales, plus the bias, in f64 */
            for (int i = 0; i < J->k; i++) xr[i] = (double)or_e4m3_to_f32(J->x8[r * J->k + i]);
            for (int c = 0; c < J->n; c++) {
                const uint8_t* wc = J->w8 + (int64_t)c * J->k;
                double acc = 0.0;
                for (int i = 0; i < J->k; i++) acc += xr[i] * (double)or_e4m3_to_f32(wc[i]);
                acc *= (double)J->x_scale[r];
                acc *= (double)J->w_scale[c];
                y[c] = acc + (J->bias ? (double)or_bf16_to_f32(J->bias[c]) : 0.0);
            }
        } else {
            for (int i = 0; i < J->k; i++) xr[i] = (double)or_bf16_to_f32(J->x[r * J->k + i]);
            for (int c = 0; c < J->n; c++) {
                const uint16_t* wc = J->w + (int64_t)c * J->k;
                double acc = 0.0;
                for (int i = 0; i < J->k; i++) acc += xr[i] * (double)or_bf16_to_f32(wc[i]);
                y[c] = acc + (J->bias ? (double)or_bf16_to_f32(J->bias[c]) : 0.0);
            }
        }
        const int d = J->d, tok = (int)(r % J->tokens), half = J->rope_half;
        for (int part = 0; part < 3; part++) {
            const int heads = part == 0 ? J->hq : J->hkv;
            const int c0 = part == 0 ? 0 : (part == 1 ? J->hq * d : (J->hq + J->hkv) * d);
            float* out = part == 0 ? J->q : (part == 1 ? J->kk : J->v);
            for (int h = 0; h < heads; h++) {
                const double* src = y + c0 + h * d;
                float* dst = out + (r * heads + h) * (int64_t)d;
                for (int e = 0; e < d; e++) {
                    double val = src[e];
                    if (J->rope && part < 2) {
                        const int pair = (e / (2 * half)) * half + (e & (half - 1));
                        const float* cs = J->rope + ((int64_t)(tok % J->frame_len) * (d / 2) + pair) * 2;
                        const double p = src[e ^ half];
                        val = (e & half) ? src[e] * (double)cs[0] + p * (double)cs[1]
                                         : src[e] * (double)cs[0] - p * (double)cs[1];
                    }
                    dst[e] = (float)val;
                }
            }
        }
    }
    free(y);
    free(xr);
    return NULL;
}

static void qkv_run(qkv_job* jp, int nthreads) {
    qkv_job J = *jp;
    pthread_mutex_init(&J.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, qkv_worker, &J);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&J.mu);
}

void or_qkv_reference(const uint16_t* x, const uint16_t* w, const uint16_t* bias, const float* rope, int rope_half,
                      int frame_len, int m, int n, int k, int tokens, int hq, int hkv, int d, int nthreads, float* q,
                      float* kk, float* v) {
    qkv_job J;
    memset(&J, 0, sizeof J);
    J.x = x; J.w = w; J.bias = bias; J.rope = rope; J.rope_half = rope_half; J.frame_len = frame_len;
    J.m = m; J.n = n; J.k = k; J.tokens = tokens; J.hq = hq; J.hkv = hkv; J.d = d;
    J.q = q; J.kk = kk; J.v = v;
    qkv_run(&J, nthreads);
}

void or_qkv_reference_fp8(const uint8_t* x8, const float* x_scale, const uint8_t* w8, const float* w_scale,
                          const uint16_t* bias, const float* rope, int rope_half, int frame_len, int m, int n, int k,
                          int tokens, int hq, int hkv, int d, int nthreads, float* q, float* kk, float* v) {
    qkv_job J;
    memset(&J, 0, sizeof J);
    J.x8 = x8; J.x_scale = x_scale; J.w8 = w8; J.w_scale = w_scale;
    J.bias = bias; J.rope = rope; J.rope_half = rope_half; J.frame_len = frame_len;
    J.m = m; J.n = n; J.k = k; J.tokens = tokens; J.hq = hq; J.hkv = hkv; J.d = d;
    J.q = q; J.kk = kk; J.v = v;
    qkv_run(&J, nthreads);
}

/* ------------------------------------------------------------------ LayerNorm -> FP8 */

/* norm.cu:37-137 (Quant::PerToken, no residual branch) in f32, in the
 * kernel's order: lane l of a warp sums its chunks l, l+32, ... (8 channels
 * each) in order, the 32 lane sums meet in a xor butterfly (16, 8, 4, 2, 1);
 * mean = sum * (1/C); the variance the same way with fmaf(d, d, ss); rstd =
 * 1/sqrtf(fmaf(var_sum, 1/C, eps)) -- the kernel's rsqrtf is an
 * approximation, so rstd, and through it y and q, may differ in the last
 * place; y = fmaf((v - mean) * rstd, gamma, beta); scale = amax / 448 (1 for
 * a zero row); q = e4m3(y * (448 / amax)). */
static float lane_tree(const float* lane_vals) {
    float v[32];
    memcpy(v, lane_vals, sizeof v);
    for (int o = 16; o > 0; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ o];
        memcpy(v, t, sizeof v);
    }
    return v[0];
}

void or_layer_norm_fp8(const void* x, int x_f32, int64_t rows, int c, const float* gamma, const float* beta, float eps,
                       uint16_t* out, uint8_t* q8, float* scales) {
    const int nch = c / 256;
    float* v = (float*)malloc(sizeof(float) * (size_t)c);
    for (int64_t r = 0; r < rows; r++) {
        for (int i = 0; i < c; i++)
            v[i] = x_f32 ? ((const float*)x)[r * c + i] : or_bf16_to_f32(((const uint16_t*)x)[r * c + i]);
        float ls[32];
        for (int l = 0; l < 32; l++) {
            float s = 0.0f;
            for (int i = 0; i < nch; i++)
                for (int j = 0; j < 8; j++) s += v[(i * 32 + l) * 8 + j];
            ls[l] = s;
        }
        const float mean = lane_tree(ls) * (1.0f / (float)c);
        for (int l = 0; l < 32; l++) {
            float ss = 0.0f;
            for (int i = 0; i < nch; i++)
                for (int j = 0; j < 8; j++) {
                    const float d = v[(i * 32 + l) * 8 + j] - mean;
                    ss = fmaf(d, d, ss);
                }
            ls[l] = ss;
        }
        const float rstd = 1.0f / sqrtf(fmaf(lane_tree(ls), 1.0f / (float)c, eps));
        float amax = 0.0f;
        for (int i = 0; i < c; i++) {
            v[i] = fmaf((v[i] - mean) * rstd, gamma[i], beta[i]);
            if (fabsf(v[i]) > amax) amax = fabsf(v[i]);
            if (out) out[r * c + i] = or_f32_to_bf16(v[i]);
        }
        const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
        scales[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
        for (int i = 0; i < c; i++) q8[r * c + i] = or_f32_to_e4m3(v[i] * inv);
    }
    free(v);
}

/* ------------------------------------------------------------------ rows -> FP8 */

/* norm.cu:170-229 (Quant::PerToken, no activation): v = y * tok * chan +
 * bias (separate roundings), amax over the row (order-free), scale =
 * amax / 448 (1 for a zero row), q = e4m3(v * (448 / amax)).  Exact. */
void or_rows_fp8(const uint16_t* y, int64_t rows, int c, int64_t ld, const float* tok, const float* chan,
                 const uint16_t* bias, uint8_t* q8, float* scales) {
    float* v = (float*)malloc(sizeof(float) * (size_t)c);
    for (int64_t r = 0; r < rows; r++) {
        const float ts = tok ? tok[r] : 1.0f;
        float amax = 0.0f;
        for (int i = 0; i < c; i++) {
            float x = or_bf16_to_f32(y[r * ld + i]) * ts;
            if (chan) x = x * chan[i];
            if (bias) x = x + or_bf16_to_f32(bias[i]);
            v[i] = x;
            if (fabsf(x) > amax) amax = fabsf(x);
        }
        const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
        scales[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
        for (int i = 0; i < c; i++) q8[r * c + i] = or_f32_to_e4m3(v[i] * inv);
    }
    free(v);
}
