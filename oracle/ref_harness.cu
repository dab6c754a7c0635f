// Launcher for the reference's own SageAttention2 kernels -- TEST
// INFRASTRUCTURE ONLY (a GPU oracle; never linked into the product).
//
// oracle/Makefile concatenates the reference's header-free CUDA sources
// (platform/spl-nn/cuda/sage_common.cu, sage_quant.cu, sage_attn.cu, as
// src/sage/mod.rs:85-94 does for NVRTC) into oracle/_ref/sage_ref_src.cu and
// compiles this file once per head dim with the tile defines of
// src/sage/mod.rs:126-141.  The entry point fills SgGeom the way
// SageAttention::prepare does (mod.rs:710-768) and launches sg_prep,
// sg_finalize, sg_quant_kv and sg_attn_{dense,merge} with the grids of
// mod.rs:789-870.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include REF_SRC

#include <stddef.h>

// The struct the reference's Rust host passes by value (its Geom, checked by
// src/sage/tests.rs:234-242): 12 i64 strides, 16 i32, 3 f32 and padding.
// This harness fills it field by field, so the same layout pins that the
// reference kernels read what the harness wrote.
static_assert(sizeof(SgGeom) == 12 * 8 + 16 * 4 + 4 * 4, "SgGeom size");
static_assert(offsetof(SgGeom, batch) == 96, "SgGeom.batch offset");
static_assert(offsetof(SgGeom, flags) == 96 + 15 * 4, "SgGeom.flags offset");
static_assert(offsetof(SgGeom, q_mul) == 96 + 16 * 4, "SgGeom.q_mul offset");
static_assert(offsetof(SgGeom, v_range) == 96 + 18 * 4, "SgGeom.v_range offset");

static int g_smem_set = 0;

extern "C" int ref_head_dim(void) { return SG_D; }

// strides[12]: q (batch, token, head), k, v, out -- bf16 elements.
// dims[10]: batch, heads, tokens, merge stride (1 dense), frames, special,
//           grid_h, grid_w, dense_frames, flags.
// Returns 0 or a cudaError_t.
extern "C" int ref_sage_run(const void* q, const void* k, const void* v, const float* ln, const long long* strides,
                            const int* dims, float q_mul, float ln_eps, float v_range, void* q8, float* q_scale,
                            void* k8, float* k_scale, void* v8, float* stats, float* kbias, float* part, void* out,
                            void* stream_ptr) {
    cudaStream_t st = (cudaStream_t)stream_ptr;
    SgGeom g;
    memset(&g, 0, sizeof(g));
    g.q_sb = strides[0]; g.q_st = strides[1]; g.q_sh = strides[2];
    g.k_sb = strides[3]; g.k_st = strides[4]; g.k_sh = strides[5];
    g.v_sb = strides[6]; g.v_st = strides[7]; g.v_sh = strides[8];
    g.o_sb = strides[9]; g.o_st = strides[10]; g.o_sh = strides[11];
    const int batch = dims[0], heads = dims[1], tokens = dims[2], s = dims[3];
    g.batch = batch;
    g.heads = heads;
    g.tokens = tokens;
    g.tq_pad = (tokens + SG_QTILE - 1) / SG_QTILE * SG_QTILE;
    g.merge = s;
    g.frames = s > 1 ? dims[4] : 1;
    g.special = s > 1 ? dims[5] : 0;
    g.grid_h = s > 1 ? dims[6] : 0;
    g.grid_w = s > 1 ? dims[7] : 0;
    const int dense_frames = s > 1 ? (dims[8] < dims[4] ? dims[8] : dims[4]) : 0;
    g.dense_frames = dense_frames;
    g.frame_tokens = g.special + g.grid_h * g.grid_w;
    g.merged_frame = s > 1 ? g.special + ((g.grid_h + s - 1) / s) * ((g.grid_w + s - 1) / s) : 0;
    g.merged_w = s > 1 ? (g.grid_w + s - 1) / s : 0;
    g.tk = s > 1 ? dense_frames * g.frame_tokens + (g.frames - dense_frames) * g.merged_frame : tokens;
    g.tk_pad = (g.tk + SG_KBLOCK - 1) / SG_KBLOCK * SG_KBLOCK;
    g.q_tiles = g.tq_pad / SG_QTILE;
    g.flags = dims[9];
    g.q_mul = q_mul;
    g.ln_eps = ln_eps;
    g.v_range = v_range;

    sg_prep<<<dim3(g.q_tiles, heads, batch), 256, 0, st>>>((const sg_u16*)q, (const sg_u16*)k, (const sg_u16*)v, ln,
                                                           (sg_i8*)q8, q_scale, part, g);
    sg_finalize<<<dim3(heads, batch), 256, 0, st>>>(part, stats, g);
    sg_quant_kv<<<dim3(g.tk_pad / SG_KBLOCK, heads, batch), 256, 0, st>>>(
        (const sg_u16*)k, (const sg_u16*)v, ln, stats, (sg_i8*)k8, k_scale, (sg_u8*)v8, kbias, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    if (out) {
        const int smem = SG_BM * SG_D + SG_STAGES * 2 * SG_KBLOCK * SG_D;
        if (!g_smem_set) {
            cudaFuncSetAttribute(sg_attn_dense, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            cudaFuncSetAttribute(sg_attn_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            g_smem_set = 1;
        }
        dim3 grid(g.tq_pad / SG_BM, heads, batch);
        if (s > 1)
            sg_attn_merge<<<grid, SG_NW * 32, smem, st>>>((const sg_i8*)q8, q_scale, (const sg_i8*)k8, k_scale,
                                                          (const sg_u8*)v8, stats, kbias, (sg_u16*)out, g);
        else
            sg_attn_dense<<<grid, SG_NW * 32, smem, st>>>((const sg_i8*)q8, q_scale, (const sg_i8*)k8, k_scale,
                                                          (const sg_u8*)v8, stats, kbias, (sg_u16*)out, g);
        e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
    }
    return 0;
}

// Attention only, on buffers a previous ref_sage_run filled (for timing the
// reference kernel alone).  Same arguments as ref_sage_run.
extern "C" int ref_sage_attend(const long long* strides, const int* dims, float q_mul, float v_range, const void* q8,
                               const float* q_scale, const void* k8, const float* k_scale, const void* v8,
                               const float* stats, const float* kbias, void* out, void* stream_ptr) {
    cudaStream_t st = (cudaStream_t)stream_ptr;
    SgGeom g;
    memset(&g, 0, sizeof(g));
    g.o_sb = strides[9]; g.o_st = strides[10]; g.o_sh = strides[11];
    const int batch = dims[0], heads = dims[1], tokens = dims[2], s = dims[3];
    g.batch = batch;
    g.heads = heads;
    g.tokens = tokens;
    g.tq_pad = (tokens + SG_QTILE - 1) / SG_QTILE * SG_QTILE;
    g.merge = s;
    if (s > 1) {
        g.frames = dims[4];
        g.special = dims[5];
        g.grid_h = dims[6];
        g.grid_w = dims[7];
        g.dense_frames = dims[8] < dims[4] ? dims[8] : dims[4];
        g.frame_tokens = g.special + g.grid_h * g.grid_w;
        g.merged_frame = g.special + ((g.grid_h + s - 1) / s) * ((g.grid_w + s - 1) / s);
        g.tk = g.dense_frames * g.frame_tokens + (g.frames - g.dense_frames) * g.merged_frame;
    } else {
        g.tk = tokens;
    }
    g.tk_pad = (g.tk + SG_KBLOCK - 1) / SG_KBLOCK * SG_KBLOCK;
    g.q_tiles = g.tq_pad / SG_QTILE;
    g.q_mul = q_mul;
    g.v_range = v_range;
    const int smem = SG_BM * SG_D + SG_STAGES * 2 * SG_KBLOCK * SG_D;
    if (!g_smem_set) {
        cudaFuncSetAttribute(sg_attn_dense, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaFuncSetAttribute(sg_attn_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        g_smem_set = 1;
    }
    dim3 grid(g.tq_pad / SG_BM, heads, batch);
    if (s > 1)
        sg_attn_merge<<<grid, SG_NW * 32, smem, st>>>((const sg_i8*)q8, q_scale, (const sg_i8*)k8, k_scale,
                                                      (const sg_u8*)v8, stats, kbias, (sg_u16*)out, g);
    else
        sg_attn_dense<<<grid, SG_NW * 32, smem, st>>>((const sg_i8*)q8, q_scale, (const sg_i8*)k8, k_scale,
                                                      (const sg_u8*)v8, stats, kbias, (sg_u16*)out, g);
    return (int)cudaGetLastError();
}
