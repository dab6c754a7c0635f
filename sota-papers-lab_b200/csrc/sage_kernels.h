// Internal interface between the C-ABI host code (sage_api.cpp) and the
// CUDA translation units.  Not installed; the public ABI is include/splsage.h.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sp {

// Geometry of one prepare/attend call.  Strides are in bf16 elements.
// Mirrors the reference's SgGeom (platform/spl-nn/cuda/sage_common.cu:39-64)
// plus kv_heads and the causal flag, which the reference does not have.
struct Geom {
    long long q_sb, q_st, q_sh;
    long long k_sb, k_st, k_sh;
    long long v_sb, v_st, v_sh;
    long long o_sb, o_st, o_sh;
    int batch, heads, kv_heads, tokens;
    int tq_pad, tk, tk_pad, q_tiles;
    int merge, frames, frame_tokens, special;
    int grid_h, grid_w, merged_frame, merged_w;
    int dense_frames, flags, causal, pad0;
    float q_mul, ln_eps, v_range, pad1;
    // Segment attention (context parallelism): the query tiles start at
    // tile q_tile0 of the workspace's Q, the keys at key k_key0 of the K/V
    // buffer; tk is then the segment's key count.  Both 0 otherwise.
    // cp_first: the segment is the first of its query rows (acc and lse are
    // written, not merged into).
    int q_tile0, k_key0, cp_first;
    // Persistent kernels launch at most this many CTAs (0: one per SM).
    int max_ctas;
    // Causal attention over gathered keys (context parallelism by
    // all-gather): the keys are the whole sequence in order and the
    // workspace's query rows are two chunks of it, local rows [0, q_split)
    // at global rows q_goff0 + i and rows [q_split, tokens) at q_goff1 +
    // (i - q_split); local row i sees global keys 0 .. its global row.
    // q_split = 0: queries and keys share positions (the plain causal mask).
    int q_split, q_goff0, q_goff1;
};

// Device buffers of one workspace.  Layouts (b = batch, h = q head,
// g = kv head):
//   q8      i8  [b][h][tq_pad][D]         (reference layout)
//   q_scale f32 [b][h][tq_pad/16]         (reference layout)
//   k8      i8  [b][g][tk_pad][D]         (reference layout)
//   k_scale f32 [b][g][tk_pad/64]         (reference layout)
//   v8      u8  [b][g][D][tk_pad]         E4M3, channel-major, keys in order:
//                                         the K-major B operand of the PV UMMA
//   stats   f32 [b][g][4][D]              (reference layout)
//   kbias   f32 [tk_pad]                  log2(count) or -inf (merge only)
//   part    f32 [b][g][q_tiles][4][D]     per-tile channel statistics
//   err     u32 [1]                       device error word
// Launches kern with programmatic stream serialization: it may start while
// the previous kernel on the stream finishes; it must call griddep_wait
// before it reads anything that kernel writes.
template <typename... Params, typename... Args>
inline cudaError_t launch_after_previous(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem,
                                         cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, ((Params)args)...);
}

struct Buffers {
    int8_t* q8;
    float* q_scale;
    int8_t* k8;
    float* k_scale;
    uint8_t* v8;
    float* stats;
    float* kbias;
    float* part;
    uint32_t* err;
    // per (batch, kv head), the statistics tiles sp_prep has finished in the
    // current launch (zero between launches: the CTA that finishes a slice's
    // last tile reduces the slice's statistics and clears its count);
    // nullptr: sp_finalize reduces them in a launch of its own.
    uint32_t* tiles_done;
};

// TMA descriptors for the attention kernel (built once per workspace).
struct AttnMaps {
    CUtensorMap q;  // q8 as {D, tq_pad, b*h}, box {D, 128, 1}
    CUtensorMap k;  // k8 as {D, tk_pad, b*g}, box {D, 128, 1}
    CUtensorMap v;  // v8 as {tk_pad, D, b*g}, box {128, D, 1}
};

// Fused QKV projection: y[m][n] = x[m][k] w[n][k]^T (+ bias[n]); columns
// [0, hq*D) are q heads, then hkv k heads, then hkv v heads.  Rows are
// (batch item, token) with `tokens` tokens per batch item.
struct QkvGeom {
    int m, n, k, tokens;
    int hq, hkv, frame_len, rope_half;
    int max_ctas;  // persistent CTAs at most (0: one per SM)
    // Q quantised in the epilogue (spl_sage_qkv_gemm_quant; nullptr: not):
    // q8 i8 [b][hq][tq_pad][D] and q_scale f32 [b][hq][tq_pad/16], the
    // workspace layouts, from the bf16-rounded Q exactly as sp_prep would.
    int8_t* q8;
    float* q_scale;
    int tq_pad;
    float q_mul;
};

struct QkvMaps {
    CUtensorMap x;  // bf16 {k, m}, box {64, 128} (E4M3: box {128, 128})
    CUtensorMap w;  // bf16 {k, n}, box {64, 256} (E4M3: box {128, 256})
};

cudaError_t launch_qkv_gemm(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope, uint16_t* q,
                            uint16_t* k, uint16_t* v, uint32_t* err, const QkvGeom& g, cudaStream_t st);
// E4M3 operands, x_scale [m] and w_scale [n] (qkv_gemm.cu).
cudaError_t launch_qkv_gemm_fp8(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                uint32_t* err, const QkvGeom& g, cudaStream_t st);
// The same GEMM on SM pairs (qkv_gemm2sm.cu): W's tensor map has a box of
// 128 rows (each CTA of a pair loads half of a 256-channel tile).
cudaError_t launch_qkv_gemm_2sm(int d, bool fp8, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                uint32_t* err, const QkvGeom& g, cudaStream_t st);
int qkv_smem_bytes();

// LayerNorm -> per-token E4M3 (layer_norm.cu): x f32 or bf16 [rows][c].
bool layer_norm_width_ok(long long c);
cudaError_t launch_layer_norm_fp8(const void* x, bool xf32, long long c, const float* gamma, const float* beta,
                                  float eps, int rows, uint16_t* out, uint8_t* q8, float* qscale, cudaStream_t st);
// bf16 rows -> per-token E4M3 (layer_norm.cu): y [rows][ld], c = 1024 * n.
cudaError_t launch_rows_fp8(const uint16_t* y, long long ld, long long c, int rows, const float* tok,
                            const float* chan, const uint16_t* bias, uint8_t* q8, float* qscale, cudaStream_t st);

// Fixed device scratch of spl_sage_quantize_noalloc (sage_quant.cu).
cudaError_t noalloc_part_buffer(float** out);
size_t noalloc_part_capacity();

// The quantiser without its Q role (Q already quantised by the QKV GEMM's
// epilogue): K/V statistics, finalize, K/V quantisation.
cudaError_t launch_prepare_kv(int d, const void* k, const void* v, const float* ln, const Buffers& buf,
                              const Geom& g, cudaStream_t st);
cudaError_t launch_prepare(int d, const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                           const Geom& g, cudaStream_t st);
cudaError_t launch_export_v(int d, const Buffers& buf, const Geom& g, uint8_t* v8_ref, cudaStream_t st);
// Context parallelism (sage_quant.cu): Q quantised and this rank's raw K/V
// channel statistics raw [b][g][4][D] = {sum K, sum V, -min V, max V};
// then, from the raw statistics combined over all ranks (sums added, the
// other two maxed), the workspace stats for `total` tokens and this rank's
// K/V quantised into buf.k8 / k_scale / v8; and the fp32 accumulator of
// segment attention converted to bf16.
cudaError_t launch_cp_prepare(int d, const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                              const Geom& g, float* raw, cudaStream_t st);
cudaError_t launch_cp_quant_kv(int d, const void* k, const void* v, const float* ln, const Buffers& buf,
                               const Geom& g, const float* raw, float total, cudaStream_t st);
cudaError_t launch_cp_finish(int d, const float* acc, const Geom& g, void* out, cudaStream_t st);
// raw [bg][4][D] = sums from rsum (entries 0-1), maxima from rmax (2-3).
cudaError_t launch_cp_merge_stats(const float* rsum, const float* rmax, float* raw, int bg, int d, cudaStream_t st);
// Segment attention merged into acc f32 (strides g.o_*) and lse f32
// [b][h][tokens] (log2 of the row's softmax denominator) by log-sum-exp.
cudaError_t launch_attend_partial(int d, const AttnMaps& maps, const Buffers& buf, const Geom& g, float* acc,
                                  float* lse, cudaStream_t st);

// launch_attend with g.q_split set: causal attention of the workspace's two
// query chunks over gathered keys (their maps in `maps`, k_scale in buf).
cudaError_t launch_attend(int d, const AttnMaps& maps, const Buffers& buf, const Geom& g, void* out,
                          cudaStream_t st);
cudaError_t attn_func_attributes(int d, int merge, int* regs, int* local_bytes);
cudaError_t launch_wait_probe(uint32_t* err, uint32_t site, unsigned long long* out, cudaStream_t st);
cudaError_t launch_peak(int kind, int n, int iters, int sms, uint32_t* err, unsigned long long* cycles,
                        cudaStream_t st);
int attn_smem_bytes(int d);

}  // namespace sp
