// Fused QKV projection for sm_100a: y = x W^T (+ bias) on the tcgen05 tensor
// cores (kind::f16, BF16 x BF16 -> FP32 in TMEM), with the QKV prologue in the
// epilogue: split q | k | v, bias, round to bf16 (the reference's GEMM writes
// bf16: platform/spl-nn/src/gemm.rs:408-416), RoPE on q and k from a
// (cos, sin) table with the reference's pairing rule
// (platform/spl-nn/cuda/qkv.cu:102-119: the partner of channel d is d ^ half,
// pair (d / 2half) * half + d % half), round to bf16 again (qkv.cu:121-133),
// and write Q, K, V in [B][T][H][D] for the quantiser.
//
// FP8 variant (the reference's FP8 block, apps/image-to-3d/src/vggt/trunk/
// block.rs:353-395: Gemm::linear_fp8 with deferred weight scales,
// platform/spl-nn/src/gemm.rs:294-337, then QkvPrologue::run with per-token
// and per-channel scales): x and w E4M3, tcgen05 kind::f8f6f4 (FP32
// accumulate, twice the BF16 rate); the epilogue rounds the accumulator to
// bf16 (the GEMM's bf16 output), multiplies by the token's activation scale
// and the channel's weight scale and adds the bias in that order
// (cuda/qkv.cu:55-73), then RoPE and bf16 as above.
//
// Tile: 128 rows x 256 output channels (two heads of 128 or four of 64), K in
// 128-byte blocks (64 bf16 or 128 E4M3 elements) through a 4-stage TMA ring.
// Persistent: one
// CTA per SM works through the output tiles in turn, with two TMEM
// accumulators (2 x 256 columns), so the epilogue of one tile overlaps the
// MMAs of the next.  Warp 0 loads, warp 1 issues the MMAs (4 x M128 N256 K16
// per block; 4 x K32 for E4M3) and owns TMEM, warps 4-7 run the epilogue,
// one thread per row.
#include <atomic>

#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

namespace gemm {
constexpr int BM = 128, BN = 256, BK_BYTES = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK_BYTES, B_BYTES = BN * BK_BYTES, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
constexpr int NTHREADS = 256;
}  // namespace gemm

// HALF: distance between the two channels of a RoPE pair (0: no RoPE).
// FP8: E4M3 operands with x_scale [m] and w_scale [n] (else BF16, unused);
// NULL scales leave the bf16 accumulator unscaled (the reference's deferred
// weight scales, applied by the consumer).
template <int D, int HALF, bool FP8>
__global__ void __launch_bounds__(gemm::NTHREADS, 1)
    sp_qkv_gemm(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                const uint16_t* __restrict__ bias, const float2* __restrict__ rope, const float* __restrict__ x_scale,
                const float* __restrict__ w_scale, uint16_t* __restrict__ q_out, uint16_t* __restrict__ k_out,
                uint16_t* __restrict__ v_out, uint32_t* __restrict__ err, const QkvGeom g) {
    using namespace gemm;
    constexpr uint32_t IDESC =
        FP8 ? make_idesc(C_F32, F_E4M3, F_E4M3, BM, BN) : make_idesc(C_F32, F_BF16, F_BF16, BM, BN);
    constexpr int BK = FP8 ? BK_BYTES : BK_BYTES / 2;  // K elements per ring stage
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t tmem_base_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_tiles = g.n / BN, ntiles = n_tiles * ((g.m + BM - 1) / BM);
    // channels from one RoPE pair row to the next (HALF = 0, no RoPE: unused)
    constexpr int PAIR_SPAN = HALF > 0 ? 2 * HALF : 1;
    const int kblocks = (g.k + BK - 1) / BK;
    // the CTA's it-th tile; consecutive tiles share their rows of x
    auto tile_m0 = [&](int t) { return (t / n_tiles) * BM; };
    auto tile_n0 = [&](int t) { return (t % n_tiles) * BN; };
    const uint32_t sbase = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    auto bar = [](uint64_t& x) { return smem_u32(&x); };

    if (tid == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(bar(full[i]), 1);
            mbar_init(bar(empty[i]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(acc_full[i]), 1);
            mbar_init(bar(acc_empty[i]), 4);
        }
        mbar_init(bar(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_base_s), 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&map_x);
            tma_prefetch_desc(&map_w);
            int issued = 0;  // k-blocks over all of this CTA's tiles
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int m0 = tile_m0(t), n0 = tile_n0(t);
                for (int kb = 0; kb < kblocks; kb++) {
                    const int s = issued % STAGES;
                    if (issued >= STAGES && !mbar_wait(bar(empty[s]), ((issued / STAGES) - 1) & 1, err, 40)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + s * STAGE_BYTES, sb = sa + A_BYTES;
                    mbar_expect_tx(bar(full[s]), STAGE_BYTES);
                    tma_load_2d(sa, &map_x, bar(full[s]), kb * BK, m0);
                    tma_load_2d(sb, &map_w, bar(full[s]), kb * BK, n0);
                    issued++;
                }
            }
            for (int s = 0; s < STAGES && s < issued; s++) {
                const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
                mbar_wait(bar(full[s]), (last / STAGES) & 1, err, 41, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int used = 0;  // k-blocks over all of this CTA's tiles
            for (int t = blockIdx.x, it = 0; t < ntiles && ok; t += gridDim.x, it++) {
                const int ab = it & 1;
                // accumulator ab is free once the epilogue read tile it - 2
                if (it >= 2 && !(ok = mbar_wait(bar(acc_empty[ab]), ((it >> 1) - 1) & 1, err, 45))) break;
                tc_fence_after();
                const uint32_t acc = tmem + ab * BN;
                for (int kb = 0; kb < kblocks; kb++, used++) {
                    const int s = used % STAGES;
                    if (!(ok = mbar_wait(bar(full[s]), (used / STAGES) & 1, err, 42))) break;
                    tc_fence_after();
                    const uint32_t sa = sbase + s * STAGE_BYTES, sb = sa + A_BYTES;
                    // four MMAs of 32 bytes of K each (K16 bf16, K32 E4M3)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t da = smem_desc(sa + kk * 32, 1024, SWZ_128B);
                        const uint64_t db = smem_desc(sb + kk * 32, 1024, SWZ_128B);
                        if (FP8)
                            umma_f8(acc, da, db, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                        else
                            umma_bf16(acc, da, db, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(bar(empty[s]));
                }
                if (ok) tc_commit(bar(acc_full[ab]));
            }
            tc_commit(bar(done));
            mbar_wait(bar(done), 0, err, 43, false);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue, one thread per row
        const int r = tid - 128;
        const uint32_t lane_off = (uint32_t)((warp - 4) * 32) << 16;
        bool ok = true;
        for (int t = blockIdx.x, it = 0; t < ntiles && ok; t += gridDim.x, it++) {
            const int ab = it & 1;
            const int m0 = tile_m0(t), n0 = tile_n0(t);
            const int row = m0 + r;
            if (!(ok = warp_all_wait(bar(acc_full[ab]), (it >> 1) & 1, err, 44))) break;
            tc_fence_after();
            const uint32_t acc = tmem + lane_off + ab * BN;
            const int bb = row / g.tokens, tok = row % g.tokens;
            const float xs = FP8 && x_scale && row < g.m ? __ldg(x_scale + row) : 1.0f;
            // the row's position inside its frame selects the RoPE table row
            const float2* rt = HALF ? rope + (long long)(tok % g.frame_len) * (D / 2) : nullptr;
#pragma unroll 1
            for (int hh = 0; hh < BN / D; hh++) {
                const int c0 = n0 + hh * D;  // first output channel of this head
                // which part and head (q | k | v, each part a whole number of heads)
                int part, head;
                if (c0 < g.hq * D) {
                    part = 0;
                    head = c0 / D;
                } else if (c0 < (g.hq + g.hkv) * D) {
                    part = 1;
                    head = (c0 - g.hq * D) / D;
                } else {
                    part = 2;
                    head = (c0 - (g.hq + g.hkv) * D) / D;
                }
                float x[D];
#pragma unroll
                for (int c = 0; c < D; c += 32) {
                    uint32_t v[32];
                    tmem_ld32(acc + hh * D + c, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        float y = __uint_as_float(v[e]);
                        if (FP8) {
                            // bf16 GEMM output, then token scale, channel scale, bias
                            y = __uint_as_float(pack_bf16x2(y, 0.f) << 16);
                            y = __fmul_rn(__fmul_rn(y, xs), w_scale ? __ldg(w_scale + c0 + c + e) : 1.0f);
                            if (bias) y = __fadd_rn(y, __uint_as_float((uint32_t)bias[c0 + c + e] << 16));
                            x[c + e] = y;
                        } else {
                            if (bias) y += __uint_as_float((uint32_t)bias[c0 + c + e] << 16);
                            x[c + e] = __uint_as_float(pack_bf16x2(y, 0.f) << 16);  // the GEMM's bf16 output
                        }
                    }
                }
                if (HALF && part < 2) {
                    // each (d, d + HALF) pair shares one table entry
#pragma unroll
                    for (int d = 0; d < D; d++) {
                        if (d & HALF) continue;
                        const int pair = (d / PAIR_SPAN) * HALF + (d & (HALF - 1));
                        const float2 cs = __ldg(rt + pair);
                        const float a = x[d], b = x[d | HALF];
                        x[d] = a * cs.x - b * cs.y;
                        x[d | HALF] = b * cs.x + a * cs.y;
                    }
                }
                if (row < g.m) {
                    uint16_t* dst = (part == 0 ? q_out : part == 1 ? k_out : v_out) +
                                    ((long long)bb * g.tokens + tok) * (long long)(part == 0 ? g.hq : g.hkv) * D +
                                    (long long)head * D;
#pragma unroll
                    for (int c = 0; c < D; c += 8) {
                        uint4 w;
                        w.x = pack_bf16x2(x[c], x[c + 1]);
                        w.y = pack_bf16x2(x[c + 2], x[c + 3]);
                        w.z = pack_bf16x2(x[c + 4], x[c + 5]);
                        w.w = pack_bf16x2(x[c + 6], x[c + 7]);
                        *reinterpret_cast<uint4*>(dst + c) = w;
                    }
                }
                if (hh == BN / D - 1) {
                    // every TMEM read of the tile is done: the next tile may
                    // accumulate into ab again
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(acc_empty[ab]));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * BN);
}

template <int D, int HALF, bool FP8>
static cudaError_t qkv_t(const QkvMaps& maps, const uint16_t* bias, const float* rope, const float* x_scale,
                         const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v, uint32_t* err,
                         const QkvGeom& g, cudaStream_t st) {
    static std::atomic<unsigned> attr_set{0};  // one bit per device ordinal
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(attr_set.load(std::memory_order_acquire) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(sp_qkv_gemm<D, HALF, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             gemm::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 32) attr_set.fetch_or(1u << dev, std::memory_order_release);
    }
    static std::atomic<int> sms[32];  // SMs per device ordinal (zero until asked)
    int n_sm = dev < 32 ? sms[dev].load(std::memory_order_relaxed) : 0;
    if (n_sm <= 0) {
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (dev < 32 && n_sm > 0) sms[dev].store(n_sm, std::memory_order_relaxed);
    }
    if (n_sm <= 0) n_sm = 148;
    if (g.max_ctas > 0 && g.max_ctas < n_sm) n_sm = g.max_ctas;
    const long long ntiles = (long long)(g.n / gemm::BN) * ((g.m + gemm::BM - 1) / gemm::BM);
    dim3 grid((unsigned)(ntiles < n_sm ? ntiles : n_sm));  // persistent: one CTA per SM
    sp_qkv_gemm<D, HALF, FP8><<<grid, gemm::NTHREADS, gemm::SMEM, st>>>(maps.x, maps.w, bias, (const float2*)rope,
                                                                        x_scale, w_scale, q, k, v, err, g);
    return cudaGetLastError();
}

template <bool FP8>
static cudaError_t qkv_dispatch(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    const int half = rope ? g.rope_half : 0;
    if (d == 64) {
        if (half == 0) return qkv_t<64, 0, FP8>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        if (half == 16) return qkv_t<64, 16, FP8>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        if (half == 32) return qkv_t<64, 32, FP8>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        return cudaErrorInvalidValue;
    }
    if (half == 0) return qkv_t<128, 0, FP8>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
    if (half == 64) return qkv_t<128, 64, FP8>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
    return cudaErrorInvalidValue;
}

// RoPE pairings: none; D=64 with pairs (i, i+16) in each 32-wide half (VGGT
// 2-D) or (i, i+32) (DINOv3); D=128 with (i, i+64) (rotate-half, Llama).
cudaError_t launch_qkv_gemm(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope, uint16_t* q,
                            uint16_t* k, uint16_t* v, uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    return qkv_dispatch<false>(d, maps, bias, rope, nullptr, nullptr, q, k, v, err, g, st);
}

cudaError_t launch_qkv_gemm_fp8(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    return qkv_dispatch<true>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
}

int qkv_smem_bytes() { return gemm::SMEM; }

}  // namespace sp
