/*
 * CPU oracle for the SageAttention2 hot path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker the tests, __graft_entry__.smoke() and the
 * bench's cpu_baseline / reference arm compare the CUDA path against.  The
 * product (libsplsage.so) never links, loads or calls it.
 *
 * It restates, in plain C, the reference's algorithm for this path:
 *   - bf16 / FP8 E4M3 codecs, the V key permutation, the KV-merge geometry,
 *     LayerNorm, f64 attention, error metrics and the SplitMix64 RNG of
 *     platform/spl-nn/src/sage/reference.rs:8-254;
 *   - the quantiser kernels sg_prep / sg_finalize / sg_quant_kv of
 *     platform/spl-nn/cuda/sage_quant.cu:59-326, bit for bit: the same
 *     reduction trees for the K/V channel sums, the same FMA contractions
 *     nvcc applies to that source, the same rounding (rint-to-even, E4M3
 *     RNE satfinite);
 *   - the quantised attention math of platform/spl-nn/cuda/sage_attn.cu
 *     (exp2 softmax, P scaled to 448 and rounded to E4M3, per-channel V
 *     dequantisation), evaluated exactly (no online rescaling), as an
 *     emulation reference.
 *
 * Extensions the reference does not have (causal mask, separate KV head
 * count for GQA) follow the usual definitions and are marked as such.
 */
#ifndef SAGE_ORACLE_H
#define SAGE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Flags of the quantiser; the values of platform/spl-nn/src/sage/mod.rs:79-82. */
#define OR_LN_Q 1
#define OR_LN_K 2
#define OR_SMOOTH_K 4
#define OR_SMOOTH_V 8

#define OR_QGROUP 16
#define OR_QTILE 128
#define OR_KBLOCK 64

/* Geometry of one quantiser call: the fields of SgGeom
 * (platform/spl-nn/cuda/sage_common.cu:39-64) plus kv_heads and d.  Strides
 * are in bf16 elements; q uses q_*, k and v their own.  With kv_heads ==
 * heads this is exactly the reference's geometry. */
typedef struct {
    int64_t q_sb, q_st, q_sh;
    int64_t k_sb, k_st, k_sh;
    int64_t v_sb, v_st, v_sh;
    int32_t batch, heads, kv_heads, tokens;
    int32_t tq_pad, tk, tk_pad, d;
    int32_t merge, frames, frame_tokens, special;
    int32_t grid_h, grid_w, merged_frame, merged_w;
    int32_t dense_frames, q_tiles, flags, pad0;
    float q_mul, ln_eps, v_range, pad1;
} or_geom;

/* ---- codecs (reference.rs:8-76) ---- */
float or_bf16_to_f32(uint16_t b);
uint16_t or_f32_to_bf16(float x);
float or_e4m3_to_f32(uint8_t b);
uint8_t or_f32_to_e4m3(float x);
void or_f32_to_e4m3_n(const float* x, uint8_t* out, int64_t n);
int or_vpos(int k);

/* ---- SplitMix64 (reference.rs:228-254) ---- */
uint64_t or_rng_next(uint64_t* state);
double or_rng_uniform(uint64_t* state);
float or_rng_normal(uint64_t* state);
/* n draws of or_rng_normal(state) * std + mean into out. */
void or_rng_normals(uint64_t* state, float* out, int64_t n, float std_, float mean);

/* Data::synthetic of platform/spl-nn/src/sage/tests.rs:300-329: clustered
 * Q/K/V [b][t][h][d], per-channel K and V offsets, outlier channels,
 * rounded to bf16.  Writes bf16 bits. */
void or_synthetic(int batch, int heads, int tokens, int d, uint64_t seed, uint16_t* q, uint16_t* k,
                  uint16_t* v);

/* ---- KV merge geometry (sage_quant.cu:210-235, reference.rs:79-107) ---- */
/* Members of merged key j: returns the count, sets the first token and the
 * row length of the cell. */
int or_members(const or_geom* g, int j, int* base, int* nx);

/* ---- the quantiser, bit-exact ---- */
/* sg_prep (sage_quant.cu:59-160): Q role for every (tile, q head, batch),
 * statistics role for every (tile, kv head, batch).  ln may be NULL when no
 * LN flag is set.  q8 [b][hq][tq_pad][d], q_scale [b][hq][tq_pad/16],
 * part [b][hkv][q_tiles][4][d]. */
void or_prep(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* ln, int8_t* q8,
             float* q_scale, float* part, const or_geom* g);
/* sg_finalize (sage_quant.cu:163-206): stats [b][hkv][4][d]. */
void or_finalize(const float* part, float* stats, const or_geom* g);
/* sg_quant_kv (sage_quant.cu:238-326): k8 [b][hkv][tk_pad][d],
 * k_scale [b][hkv][tk_pad/64], v8 in the reference layout
 * [b][hkv][tk_pad/64][d][64] with keys permuted by or_vpos, kbias [tk_pad]
 * (written only when merging). */
void or_quant_kv(const uint16_t* k, const uint16_t* v, const float* ln, const float* stats, int8_t* k8,
                 float* k_scale, uint8_t* v8, float* kbias, const or_geom* g);
/* The three in sequence (SageAttention::prepare, mod.rs:673-836).  part
 * must hold b*hkv*q_tiles*4*d floats. */
void or_prepare(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* ln, int8_t* q8,
                float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8, float* stats, float* kbias,
                float* part, const or_geom* g);

/* ---- attention ---- */
/* f64 softmax attention for one (batch, head): q [tq][d], k, v [tk][d];
 * bias_log2 adds ln2 * b_j to key j's logit (may be NULL).  causal (an
 * extension) keeps key j only for j <= i + causal_offset.  out [tq][d].
 * reference.rs:148-184. */
void or_attention_f64(const float* q, const float* k, const float* v, const float* bias_log2, int tq, int tk,
                      int d, float scale, int causal, int causal_offset, float* out);

/* f64 attention over whole [b][t][h][d] bf16 tensors (GQA maps q head h to
 * kv head h / (heads / kv_heads)), for rows [row0, row1) of every (b, h),
 * threaded over nthreads host threads.  out holds f32 [b][t][h][d] (only
 * the selected rows are written).  K/V may be merged (or_members); the
 * +log2(count) bias is then applied.  Returns 0. */
int or_attention_bthd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const or_geom* g, float scale,
                      int causal, int row0, int row1, int nthreads, float* out);

/* The reference kernel's arithmetic on the quantised tensors, evaluated
 * without online rescaling: logits x = S * q_scale * k_scale (+ kbias, in
 * log2 units), P = e4m3(448 * 2^(x - max)), l = sum of the unrounded P,
 * O = sum P8 * V8, out = O / l * v_scale + v_mean.  Inputs in the layouts
 * or_prepare writes; out f32 [b][t][hq][d], only rows [row0, row1) of every
 * (b, h) written. */
void or_sage_emulate(const int8_t* q8, const float* q_scale, const int8_t* k8, const float* k_scale,
                     const uint8_t* v8, const float* stats, const float* kbias, const or_geom* g, int causal,
                     int row0, int row1, int nthreads, float* out);

/* The kernels' online softmax, block by block: `block` 64 is the reference
 * kernel's (platform/spl-nn/cuda/sage_attn.cu:227-420), 128 this library's.
 * Same inputs and output layout as or_sage_emulate; rows [row0, row1) of
 * every (b, h).  Agrees with a kernel to rounding noise (exp2f for
 * ex2.approx, each block's PV rounded once). */
void or_sage_online(const int8_t* q8, const float* q_scale, const int8_t* k8, const float* k_scale,
                    const uint8_t* v8, const float* stats, const float* kbias, const or_geom* g, int causal,
                    int block, int row0, int row1, int nthreads, float* out);

/* The QKV path of one block in f64: y = x w^T + bias (host::linear,
 * platform/spl-nn/src/host.rs) then the QKV prologue (qkv::reference,
 * platform/spl-nn/src/qkv.rs:306-372, generalised to head dim 128 and any
 * RoPE pair distance): split q | k | v, RoPE x*cos -+ partner*sin on q and k
 * with partner d ^ rope_half and table row token % frame_len.  x bf16
 * [m][k], w bf16 [n][k], bias bf16 [n] or NULL, rope f32 [frame_len][d/2][2]
 * or NULL.  Outputs f32 q [m][hq][d], k and v [m][hkv][d]. */
void or_qkv_reference(const uint16_t* x, const uint16_t* w, const uint16_t* bias, const float* rope, int rope_half,
                      int frame_len, int m, int n, int k, int tokens, int hq, int hkv, int d, int nthreads, float* q,
                      float* kk, float* v);
/* The FP8 QKV side (gemm.rs:294-337 with deferred scales, then qkv.rs:306-372
 * with tok and chan): E4M3 x8 [m][k] with x_scale [m], w8 [n][k] with
 * w_scale [n], in f64; outputs as or_qkv_reference. */
void or_qkv_reference_fp8(const uint8_t* x8, const float* x_scale, const uint8_t* w8, const float* w_scale,
                          const uint16_t* bias, const float* rope, int rope_half, int frame_len, int m, int n, int k,
                          int tokens, int hq, int hkv, int d, int nthreads, float* q, float* kk, float* v);
/* Norm::layer_norm with Quant::PerToken (norm.cu:37-137) on the CPU, f32 in
 * the kernel's order; rstd through 1/sqrtf (the kernel's rsqrtf may differ
 * in the last place).  x f32 (x_f32 = 1) or bf16 [rows][c], c = 256 * n. */
void or_layer_norm_fp8(const void* x, int x_f32, int64_t rows, int c, const float* gamma, const float* beta, float eps,
                       uint16_t* out, uint8_t* q8, float* scales);
/* Norm::row_epilogue with Quant::PerToken, no activation (norm.cu:170-229):
 * y bf16 [rows][ld], tok [rows], chan [c], bias bf16 [c] each optional. */
void or_rows_fp8(const uint16_t* y, int64_t rows, int c, int64_t ld, const float* tok, const float* chan,
                 const uint16_t* bias, uint8_t* q8, float* scales);

/* LayerNorm of one row in f64 (reference.rs:110-118). */
void or_layer_norm(float* x, const float* w, const float* b, int n, float eps);

/* Errors::of (reference.rs:201-225): out = {cos, rel_l1, rel_l2, max_abs, ref_max}. */
void or_errors(const float* ours, const float* ref, int64_t n, double* out);

/* FLOPs of one call, 4 * B * H * Tq * Tk * D (mod.rs:905-910). */
double or_flops(int batch, int heads, int tq, int tk, int d);

#ifdef __cplusplus
}
#endif
#endif
