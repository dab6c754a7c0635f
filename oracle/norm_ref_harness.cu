// Launcher for the reference's own LayerNorm kernels -- TEST INFRASTRUCTURE
// ONLY (a GPU oracle; never linked into the product).
//
// oracle/Makefile concatenates platform/spl-nn/cuda/common.cuh and norm.cu
// the way src/norm.rs:131 does for NVRTC into oracle/_ref/norm_ref_src.cu;
// this file fills LnArgs as Norm::layer_norm does (norm.rs:171-274: no
// residual branch, Quant::PerToken) and launches ln_{f32,bf16}_c<n> with the
// grid of norm.rs:259-263 (rows / 4 blocks of 128 threads).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include REF_SRC

#define LN_CASE(N)                                                              \
    case N * 256:                                                               \
        if (x_f32)                                                              \
            ln_f32_c##N<<<blocks, 128, 0, st>>>(a);                             \
        else                                                                    \
            ln_bf16_c##N<<<blocks, 128, 0, st>>>(a);                            \
        break;

// Returns 0 or a cudaError_t (cudaErrorInvalidValue for an unsupported c).
extern "C" int ref_layer_norm_fp8(const void* x, int x_f32, int rows, int c, const float* gamma, const float* beta,
                                  float eps, void* out, void* q8, float* scales, void* stream_ptr) {
    cudaStream_t st = (cudaStream_t)stream_ptr;
    LnArgs a;
    memset(&a, 0, sizeof a);
    a.x = (unsigned long long)x;
    a.gamma = (unsigned long long)gamma;
    a.beta = (unsigned long long)beta;
    a.out = (unsigned long long)out;
    a.q = (unsigned long long)q8;
    a.qscale = (unsigned long long)scales;
    a.rows = rows;
    a.eps = eps;
    const unsigned blocks = (unsigned)((rows + 3) / 4);
    switch (c) {
        LN_CASE(1)
        LN_CASE(2)
        LN_CASE(3)
        LN_CASE(4)
        LN_CASE(6)
        LN_CASE(8)
        default: return (int)cudaErrorInvalidValue;
    }
    return (int)cudaGetLastError();
}

// Norm::row_epilogue (norm.rs:280-336) with Quant::PerToken and no
// activation: RowArgs as the host fills it, row_c<n> with one 128-thread
// block per row.
extern "C" int ref_rows_fp8(const void* y, int rows, int c, int ld, const float* tok, const float* chan,
                            const void* bias, void* q8, float* scales, void* stream_ptr) {
    cudaStream_t st = (cudaStream_t)stream_ptr;
    RowArgs a;
    memset(&a, 0, sizeof a);
    a.y = (unsigned long long)y;
    a.ytok = (unsigned long long)tok;
    a.ychan = (unsigned long long)chan;
    a.bias = (unsigned long long)bias;
    a.q = (unsigned long long)q8;
    a.qscale = (unsigned long long)scales;
    a.rows = rows;
    a.ld = ld;
    a.act = 0;
    const dim3 grid((unsigned)rows);
    switch (c) {
        case 1024: row_c1<<<grid, 128, 0, st>>>(a); break;
        case 2048: row_c2<<<grid, 128, 0, st>>>(a); break;
        case 3072: row_c3<<<grid, 128, 0, st>>>(a); break;
        case 4096: row_c4<<<grid, 128, 0, st>>>(a); break;
        default: return (int)cudaErrorInvalidValue;
    }
    return (int)cudaGetLastError();
}
