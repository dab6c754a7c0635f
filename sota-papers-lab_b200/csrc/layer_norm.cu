// LayerNorm -> FP8 E4M3 with one scale per token, the activation side of the
// reference's FP8 transformer block (apps/image-to-3d/src/vggt/trunk/
// block.rs:326-352: LN1 feeding the FP8 QKV GEMM): Norm::layer_norm with
// Quant::PerToken (platform/spl-nn/src/norm.rs:171-274, cuda/norm.cu:37-137).
//
// One warp per row, the row held in registers: lane l owns the 8-channel
// chunks l, l + 32, l + 64, ... (C = 256 * NCH).  The arithmetic is the
// reference's step for step, so that the bytes are the same: mean = warp
// sum (xor butterfly 16, 8, 4, 2, 1) of the lane sums (chunks in order,
// channels in order) times 1/C; the variance the same way over (v - mean)^2
// with the square fused into the running sum; rstd = rsqrtf(var * 1/C + eps)
// (fused multiply-add); y = ((v - mean) * rstd) * gamma + beta (fused
// multiply-add); amax over |y|, scale = amax / 448 (1 for a zero row),
// q = E4M3(y * (448 / amax)), round to nearest even, saturating.  The row is
// read once (f32 or bf16) and written once as FP8 (and as bf16 when asked):
// an HBM-bound pass.
//
// Rows wider than the reference supports (3072 and 4096 channels) would
// need ~255 registers a lane in that layout, leaving 8 warps per SM; they
// run on two warps per row instead (sp_ln_fp8_wide): warp w owns the
// chunks w * NCH/2 ... of the row, each warp reduces its lanes as above and
// the two warp sums are added in shared memory, warp 0's first.  The
// arithmetic is otherwise the same; the sums' order differs from a
// one-warp reduction in the last bits.
#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

namespace {

__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max_xor(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace

template <bool XF32, int NCH>
__global__ void __launch_bounds__(128) sp_ln_fp8(const void* __restrict__ x, const float* __restrict__ gamma,
                                                 const float* __restrict__ beta, float eps, int rows,
                                                 uint16_t* __restrict__ out, uint8_t* __restrict__ q8,
                                                 float* __restrict__ qscale) {
    constexpr int C = NCH * 256;
    const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const long long base = (long long)row * C;

    float v[NCH][8];
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        const int c0 = (i * 32 + lane) * 8;
        if (XF32) {
            const float4 a = __ldg(reinterpret_cast<const float4*>((const float*)x + base + c0));
            const float4 b = __ldg(reinterpret_cast<const float4*>((const float*)x + base + c0 + 4));
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
            v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
        } else {
            unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>((const uint16_t*)x + base + c0)), v[i]);
        }
    }

    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) s += v[i][j];
    const float mean = warp_sum_xor(s) * (1.0f / C);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float d = v[i][j] - mean;
            ss = fmaf(d, d, ss);
        }
    const float rstd = rsqrtf(fmaf(warp_sum_xor(ss), 1.0f / C, eps));

    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        const int c0 = (i * 32 + lane) * 8;
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c0));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c0 + 4));
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + c0));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + c0 + 4));
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[i][j] = fmaf((v[i][j] - mean) * rstd, g[j], b[j]);
            amax = fmaxf(amax, fabsf(v[i][j]));
        }
        if (out) {
            const uint4 w = make_uint4(pack_bf16x2(v[i][0], v[i][1]), pack_bf16x2(v[i][2], v[i][3]),
                                       pack_bf16x2(v[i][4], v[i][5]), pack_bf16x2(v[i][6], v[i][7]));
            *reinterpret_cast<uint4*>(out + base + c0) = w;
        }
    }
    amax = warp_max_xor(amax);
    const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
    if (lane == 0) qscale[row] = amax > 0.0f ? amax / 448.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        const int c0 = (i * 32 + lane) * 8;
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = v[i][j] * inv;
        const uint2 w = make_uint2(e4m3x4(t[0], t[1], t[2], t[3]), e4m3x4(t[4], t[5], t[6], t[7]));
        *reinterpret_cast<uint2*>(q8 + base + c0) = w;
    }
}

// Two warps per row, two rows per 128-thread block (see the file comment).
template <bool XF32, int NCH>
__global__ void __launch_bounds__(128) sp_ln_fp8_wide(const void* __restrict__ x, const float* __restrict__ gamma,
                                                      const float* __restrict__ beta, float eps, int rows,
                                                      uint16_t* __restrict__ out, uint8_t* __restrict__ q8,
                                                      float* __restrict__ qscale) {
    constexpr int C = NCH * 256, HALF = NCH / 2;
    __shared__ float red[2][2];  // [row in block][warp of the row]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rb = warp >> 1, w = warp & 1;  // row in the block, warp of the row
    const int row = blockIdx.x * 2 + rb;
    const bool valid = row < rows;  // every warp reaches the block barriers
    const long long base = (long long)(valid ? row : 0) * C;

    float v[HALF][8];
#pragma unroll
    for (int i = 0; i < HALF; i++) {
        const int c0 = ((w * HALF + i) * 32 + lane) * 8;
        if (XF32) {
            const float4 a = __ldg(reinterpret_cast<const float4*>((const float*)x + base + c0));
            const float4 b = __ldg(reinterpret_cast<const float4*>((const float*)x + base + c0 + 4));
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
            v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
        } else {
            unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>((const uint16_t*)x + base + c0)), v[i]);
        }
    }
    auto row_sum = [&](float part) {
        part = warp_sum_xor(part);
        if (lane == 0) red[rb][w] = part;
        __syncthreads();
        const float t = red[rb][0] + red[rb][1];
        __syncthreads();  // red is reused by the next reduction
        return t;
    };
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < HALF; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) s += v[i][j];
    const float mean = row_sum(s) * (1.0f / C);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < HALF; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float d = v[i][j] - mean;
            ss = fmaf(d, d, ss);
        }
    const float rstd = rsqrtf(fmaf(row_sum(ss), 1.0f / C, eps));

    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < HALF; i++) {
        const int c0 = ((w * HALF + i) * 32 + lane) * 8;
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c0));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c0 + 4));
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + c0));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + c0 + 4));
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[i][j] = fmaf((v[i][j] - mean) * rstd, g[j], b[j]);
            amax = fmaxf(amax, fabsf(v[i][j]));
        }
        if (out && valid) {
            const uint4 o = make_uint4(pack_bf16x2(v[i][0], v[i][1]), pack_bf16x2(v[i][2], v[i][3]),
                                       pack_bf16x2(v[i][4], v[i][5]), pack_bf16x2(v[i][6], v[i][7]));
            *reinterpret_cast<uint4*>(out + base + c0) = o;
        }
    }
    amax = warp_max_xor(amax);
    if (lane == 0) red[rb][w] = amax;
    __syncthreads();
    amax = fmaxf(red[rb][0], red[rb][1]);
    const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
    if (!valid) return;
    if (w == 0 && lane == 0) qscale[row] = amax > 0.0f ? amax / 448.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < HALF; i++) {
        const int c0 = ((w * HALF + i) * 32 + lane) * 8;
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = v[i][j] * inv;
        const uint2 q = make_uint2(e4m3x4(t[0], t[1], t[2], t[3]), e4m3x4(t[4], t[5], t[6], t[7]));
        *reinterpret_cast<uint2*>(q8 + base + c0) = q;
    }
}

template <int NCH>
static cudaError_t ln_wide_t(const void* x, bool xf32, const float* gamma, const float* beta, float eps, int rows,
                             uint16_t* out, uint8_t* q8, float* qscale, cudaStream_t st) {
    const unsigned blocks = (unsigned)((rows + 1) / 2);  // two rows (four warps) per block
    if (xf32)
        sp_ln_fp8_wide<true, NCH><<<blocks, 128, 0, st>>>(x, gamma, beta, eps, rows, out, q8, qscale);
    else
        sp_ln_fp8_wide<false, NCH><<<blocks, 128, 0, st>>>(x, gamma, beta, eps, rows, out, q8, qscale);
    return cudaGetLastError();
}

template <int NCH>
static cudaError_t ln_t(const void* x, bool xf32, const float* gamma, const float* beta, float eps, int rows,
                        uint16_t* out, uint8_t* q8, float* qscale, cudaStream_t st) {
    const unsigned blocks = (unsigned)((rows + 3) / 4);  // four rows (warps) per block
    if (xf32)
        sp_ln_fp8<true, NCH><<<blocks, 128, 0, st>>>(x, gamma, beta, eps, rows, out, q8, qscale);
    else
        sp_ln_fp8<false, NCH><<<blocks, 128, 0, st>>>(x, gamma, beta, eps, rows, out, q8, qscale);
    return cudaGetLastError();
}

bool layer_norm_width_ok(long long c) {
    return c == 256 || c == 512 || c == 768 || c == 1024 || c == 1536 || c == 2048 || c == 3072 || c == 4096;
}

cudaError_t launch_layer_norm_fp8(const void* x, bool xf32, long long c, const float* gamma, const float* beta,
                                  float eps, int rows, uint16_t* out, uint8_t* q8, float* qscale, cudaStream_t st) {
    switch (c) {
        case 256: return ln_t<1>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 512: return ln_t<2>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 768: return ln_t<3>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 1024: return ln_t<4>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 1536: return ln_t<6>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 2048: return ln_t<8>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 3072: return ln_wide_t<12>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        case 4096: return ln_wide_t<16>(x, xf32, gamma, beta, eps, rows, out, q8, qscale, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sp

namespace sp {

// Norm::row_epilogue with Quant::PerToken (platform/spl-nn/src/norm.rs:280-336,
// cuda/norm.cu:170-229): the attention output (or any bf16 GEMM output) to
// per-token E4M3 for the next FP8 GEMM (block.rs: attention output -> FP8 ->
// proj).  y bf16 [rows][ld], optional token scale, channel scale and bias
// (v = y * tok * chan + bias, in that order), amax over the row, scale =
// amax / 448 (1 for a zero row), q = E4M3(v * (448 / amax)).  One 128-thread
// block per row; thread t owns the 8-channel chunks t, t + 128, ...
// (C = 1024 * NCH); the warp maxima meet in shared memory.
template <int NCH>
__global__ void __launch_bounds__(128) sp_rows_fp8(const uint16_t* __restrict__ y, long long ld,
                                                   const float* __restrict__ tok, const float* __restrict__ chan,
                                                   const uint16_t* __restrict__ bias, uint8_t* __restrict__ q8,
                                                   float* __restrict__ qscale) {
    constexpr int C = NCH * 1024;
    __shared__ float wmax[4];
    const int row = blockIdx.x, t = threadIdx.x;
    const float ts = tok ? __ldg(tok + row) : 1.0f;
    float v[NCH][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        const int c0 = (i * 128 + t) * 8;
        unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(y + (long long)row * ld + c0)), v[i]);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float x = __fmul_rn(v[i][j], ts);
            if (chan) x = __fmul_rn(x, __ldg(chan + c0 + j));
            if (bias) x = __fadd_rn(x, __uint_as_float((uint32_t)__ldg(bias + c0 + j) << 16));
            v[i][j] = x;
            amax = fmaxf(amax, fabsf(x));
        }
    }
    amax = warp_max_xor(amax);
    if ((t & 31) == 0) wmax[t >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
    if (t == 0) qscale[row] = amax > 0.0f ? amax / 448.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        float s[8];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j] = v[i][j] * inv;
        const uint2 w = make_uint2(e4m3x4(s[0], s[1], s[2], s[3]), e4m3x4(s[4], s[5], s[6], s[7]));
        *reinterpret_cast<uint2*>(q8 + (long long)row * C + (i * 128 + t) * 8) = w;
    }
}

cudaError_t launch_rows_fp8(const uint16_t* y, long long ld, long long c, int rows, const float* tok,
                            const float* chan, const uint16_t* bias, uint8_t* q8, float* qscale, cudaStream_t st) {
    const dim3 grid((unsigned)rows);
    switch (c) {
        case 1024: sp_rows_fp8<1><<<grid, 128, 0, st>>>(y, ld, tok, chan, bias, q8, qscale); break;
        case 2048: sp_rows_fp8<2><<<grid, 128, 0, st>>>(y, ld, tok, chan, bias, q8, qscale); break;
        case 3072: sp_rows_fp8<3><<<grid, 128, 0, st>>>(y, ld, tok, chan, bias, q8, qscale); break;
        case 4096: sp_rows_fp8<4><<<grid, 128, 0, st>>>(y, ld, tok, chan, bias, q8, qscale); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sp
