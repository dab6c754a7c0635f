// The QKV GEMM of qkv_gemm.cu on SM pairs: a cluster of two CTAs computes a
// 256 x 256 output tile with tcgen05.mma.cta_group::2 (M = 256).  Each CTA
// loads its own 128 rows of x and its own 128 rows of W (TMA, no
// multicast), so a 128-byte K stage is 32 KB per CTA instead of 48 KB for
// the same work, and six stages fit where four did: at the FP8 rate the
// single-SM kernel's four 48 KB stages cover too little of the L2 latency.
//
// Roles per CTA: warp 0 loads (both CTAs' loads complete on the leader's
// stage barrier, which the leader arms for both halves), warp 1 owns TMEM
// (allocated for the pair) and, in the leader (cluster rank 0), issues the
// MMAs, whose commits arrive on the stage and accumulator barriers of both
// CTAs; the epilogue warps (4-11, or 4-7 for bf16 with K > 2048 or Q
// quantised at D = 128) read their own CTA's accumulator (rows rank * 128 +
// quarter * 32 + lane; with eight, warps 4-7 take channels 0-127 of the tile
// and warps 8-11 channels 128-255) and run the arithmetic of qkv_gemm.cu's
// epilogue (for spl_sage_qkv_gemm_quant also quantising Q to INT8 with its
// 16-row scales, so that the quantiser only reads K and V), storing through
// shared memory 64 contiguous bytes per row, then tell the leader the
// accumulator is free.  Every mbarrier wait is bounded; both CTAs always
// reach the closing cluster barrier, after which TMEM is freed.
#include <atomic>

#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

namespace gemm2 {
constexpr int BM = 128, BN = 256, BK_BYTES = 128, STAGES = 6;      // per CTA: 128 rows of the 256-row tile
constexpr int A_BYTES = BM * BK_BYTES, B_BYTES = (BN / 2) * BK_BYTES;  // each CTA holds half of B's rows
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
// each epilogue warp stages its 32 rows x 32 channels (bf16) in rows of 80
// bytes (64 + 16 of padding: conflict-free 16-byte writes), so that the
// global stores cover 64 contiguous bytes per row, 8 rows per instruction
constexpr int STG_ROW = 80, STG_WARP = 32 * STG_ROW;
constexpr int smem_bytes(int epw) { return STAGES * STAGE_BYTES + 1024 + epw * STG_WARP; }
// warps 0-3 load / MMA / idle, then EPW epilogue warps: eight where a
// tile's MMAs are short enough for a four-warp epilogue to hold them up (E4M3,
// and bf16 with K <= 2048 unless Q is quantised at D = 128, whose registers
// do not fit 384 threads), else four (C4: FP8 0.689 ms with eight, 0.722
// with four; bf16 1.184 ms with four, 1.200 with eight; C2, K = 1024: bf16
// 0.0758 ms with four, 0.0645 with eight)
constexpr int epilogue_warps(bool fp8, bool qq, int d, int k) {
    return fp8 || (k <= 2048 && !(qq && d == 128)) ? 8 : 4;  // (Q quantised at D = 128: 64 packed values per thread)
}
constexpr int nthreads(int epw) { return 128 + 32 * epw; }
}  // namespace gemm2

namespace {

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of this CTA's shared-memory word `addr` in the
// cluster's CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// Arrive once on the barrier at shared offset `bar` of both CTAs of the pair
// when this thread's tcgen05.mma so far complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            bar),
        "h"((unsigned short)3)
        : "memory");
}

template <bool FP8>
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    if (FP8)
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}"
            ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    else
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}"
            ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// TMA load into this CTA's shared memory, completing on a barrier of either
// CTA of the pair (bar: a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2 [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// Relaxed: the epilogue's accumulator reads have completed (tcgen05.wait::ld,
// then tcgen05.fence::before_thread_sync) before the arrival, and the MMA
// thread that waits on it reads nothing the epilogue writes, so no release
// of the epilogue's global stores (a wait for them to drain) is needed.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

}  // namespace

template <int D, int HALF, bool FP8, bool QQ, int EPW>
__global__ void __launch_bounds__(gemm2::nthreads(EPW), 1)
    sp_qkv_gemm_2sm(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                    const uint16_t* __restrict__ bias, const float2* __restrict__ rope,
                    const float* __restrict__ x_scale, const float* __restrict__ w_scale, uint16_t* __restrict__ q_out,
                    uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out, uint32_t* __restrict__ err,
                    const QkvGeom g) {
    using namespace gemm2;
    constexpr int TM = 2 * BM;  // rows of the pair's tile
    // channels from one RoPE pair row to the next (HALF = 0, no RoPE: unused)
    constexpr int PAIR_SPAN = HALF > 0 ? 2 * HALF : 1;
    constexpr uint32_t IDESC =
        FP8 ? make_idesc(C_F32, F_E4M3, F_E4M3, TM, BN) : make_idesc(C_F32, F_BF16, F_BF16, TM, BN);
    constexpr int BK = FP8 ? BK_BYTES : BK_BYTES / 2;  // K elements per ring stage
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t tmem_base_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int n_tiles = g.n / BN, ntiles = n_tiles * ((g.m + TM - 1) / TM);
    const int kblocks = (g.k + BK - 1) / BK;
    auto tile_m0 = [&](int t) { return (t / n_tiles) * TM; };
    auto tile_n0 = [&](int t) { return (t % n_tiles) * BN; };
    const uint32_t sbase = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    auto bar = [](uint64_t& x) { return smem_u32(&x); };

    if (tid == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(bar(full[i]), 1);   // the leader's arrival (with both CTAs' bytes)
            mbar_init(bar(empty[i]), 1);  // one commit from the leader's MMA thread
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(acc_full[i]), 1);
            mbar_init(bar(acc_empty[i]), 2 * EPW);  // epilogue warps of both CTAs
        }
        mbar_init(bar(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(&tmem_base_s), 2 * BN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    // the set-up above may overlap the end of the kernel launched before this
    // one (programmatic dependent launch); everything below reads or writes
    // memory that kernel may use
    griddep_wait();

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&map_x);
            tma_prefetch_desc(&map_w);
            int issued = 0;
            bool ok = true;
            for (int t = pair; t < ntiles && ok; t += npairs) {
                const int m0 = tile_m0(t) + (int)rank * BM, n0 = tile_n0(t) + (int)rank * (BN / 2);
                for (int kb = 0; kb < kblocks; kb++) {
                    const int s = issued % STAGES;
                    // this CTA's half of stage s is free once the pair's MMAs read it
                    if (issued >= STAGES && !mbar_wait(bar(empty[s]), ((issued / STAGES) - 1) & 1, err, 50)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + s * STAGE_BYTES, sb = sa + A_BYTES;
                    const uint32_t fb = map_to_rank(bar(full[s]), 0);  // the leader's stage barrier
                    if (leader) mbar_expect_tx(bar(full[s]), 2 * STAGE_BYTES);
                    tma_load_2d_pair(sa, &map_x, fb, kb * BK, m0);
                    tma_load_2d_pair(sb, &map_w, fb, kb * BK, n0);
                    issued++;
                }
            }
            if (leader) {
                // drain: every stage's last loads (both halves) have landed
                for (int s = 0; s < STAGES && s < issued; s++) {
                    const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
                    mbar_wait(bar(full[s]), (last / STAGES) & 1, err, 51, false);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            bool ok = true;
            int used = 0;
            for (int t = pair, it = 0; t < ntiles && ok; t += npairs, it++) {
                const int ab = it & 1;
                if (it >= 2 && !(ok = mbar_wait(bar(acc_empty[ab]), ((it >> 1) - 1) & 1, err, 55))) break;
                tc_fence_after();
                const uint32_t acc = tmem + ab * BN;
                for (int kb = 0; kb < kblocks; kb++, used++) {
                    const int s = used % STAGES;
                    if (!(ok = mbar_wait(bar(full[s]), (used / STAGES) & 1, err, 52))) break;
                    tc_fence_after();
                    const uint32_t sa = sbase + s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma_pair<FP8>(acc, smem_desc(sa + kk * 32, 1024, SWZ_128B),
                                       smem_desc(sb + kk * 32, 1024, SWZ_128B), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                    tc_commit_pair(bar(empty[s]));
                }
                if (ok) tc_commit_pair(bar(acc_full[ab]));
            }
            tc_commit_pair(bar(done));  // (the peer's copy of `done` is not waited on)
            mbar_wait(bar(done), 0, err, 53, false);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue
        // with eight epilogue warps, warps 4-7 take the tile's channels
        // 0-127 and warps 8-11 channels 128-255 (with four, warps 4-7 take
        // all); a warp reads its own TMEM lane quarter (warp % 4), one thread
        // per row.  Columns go through 32 at a time, with their RoPE partners
        // (d + HALF) when HALF >= 32, so that only 64 floats are live.
        constexpr int HEADS = (EPW == 8 ? BN / 2 : BN) / D;  // heads per epilogue warp
        const int quarter = warp & 3, chalf = EPW == 8 ? (warp - 4) >> 2 : 0;
        const int r = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        uint8_t* stg = dyn_smem + (sbase - smem_u32(dyn_smem)) + STAGES * STAGE_BYTES + (warp - 4) * STG_WARP;
        bool ok = true;
        for (int t = pair, it = 0; t < ntiles && ok; t += npairs, it++) {
            const int ab = it & 1;
            const int m0 = tile_m0(t), n0 = tile_n0(t);
            const int row = m0 + (int)rank * BM + r;
            if (!(ok = warp_all_wait(bar(acc_full[ab]), (it >> 1) & 1, err, 54))) break;
            tc_fence_after();
            const uint32_t acc = tmem + lane_off + ab * BN;
            const int bb = row / g.tokens, tok = row % g.tokens;
            const float xs = FP8 && x_scale && row < g.m ? __ldg(x_scale + row) : 1.0f;
            const float2* rt = HALF ? rope + (long long)(tok % g.frame_len) * (D / 2) : nullptr;
#pragma unroll 1
            for (int hh = chalf * HEADS; hh < (chalf + 1) * HEADS; hh++) {
                const int c0 = n0 + hh * D;
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
                // row r of q / k / v starts at r * (heads of the part) * D: the
                // flattened row index is batch * tokens + token
                const long long rstride = (long long)(part == 0 ? g.hq : g.hkv) * D;
                uint16_t* dst_head = (part == 0 ? q_out : part == 1 ? k_out : v_out) + (long long)head * D;
                // columns c .. c+31 of the head: GEMM output, scales, bias
                auto load = [&](int c, float (&x)[32]) {
                    // the bias first (independent of TMEM), so that its
                    // latency hides under the TMEM load's (hoisting the E4M3
                    // channel scales too measured slower)
                    uint4 braw[4];
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        braw[i] = bias ? __ldg(reinterpret_cast<const uint4*>(bias + c0 + c + 8 * i))
                                       : make_uint4(0, 0, 0, 0);
                    uint32_t v[32];
                    tmem_ld32(acc + hh * D + c, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e8 = 0; e8 < 32; e8 += 8) {
                        float ws[8], bs[8];
                        if (FP8 && w_scale) {
                            const float4 a = __ldg(reinterpret_cast<const float4*>(w_scale + c0 + c + e8));
                            const float4 b = __ldg(reinterpret_cast<const float4*>(w_scale + c0 + c + e8 + 4));
                            ws[0] = a.x; ws[1] = a.y; ws[2] = a.z; ws[3] = a.w;
                            ws[4] = b.x; ws[5] = b.y; ws[6] = b.z; ws[7] = b.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; e++) ws[e] = 1.0f;
                        }
                        unpack_bf16x8(braw[e8 / 8], bs);
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            float y = __uint_as_float(v[e8 + e]);
                            if (FP8) {
                                y = __uint_as_float(pack_bf16x2(y, 0.f) << 16);
                                y = __fmul_rn(__fmul_rn(y, xs), ws[e]);
                                if (bias) y = __fadd_rn(y, bs[e]);
                                x[e8 + e] = y;
                            } else {
                                // rounded to bf16 here only ahead of RoPE: the
                                // stores (and Q's quantisation) round the same way
                                if (bias) y += bs[e];
                                x[e8 + e] = HALF ? __uint_as_float(pack_bf16x2(y, 0.f) << 16) : y;
                            }
                        }
                    }
                };
                // columns c .. c+31 of the warp's 32 rows: each lane's row into
                // the staging rows, then 16 bytes per lane, 4 lanes per row
                auto store = [&](int c, const float (&x)[32]) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 w;
                        w.x = pack_bf16x2(x[e], x[e + 1]);
                        w.y = pack_bf16x2(x[e + 2], x[e + 3]);
                        w.z = pack_bf16x2(x[e + 4], x[e + 5]);
                        w.w = pack_bf16x2(x[e + 6], x[e + 7]);
                        *reinterpret_cast<uint4*>(stg + lane * STG_ROW + e * 2) = w;
                    }
                    __syncwarp();
                    const int row0 = row - lane, q16 = lane & 3;
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        const int rr = i + (lane >> 2);
                        if (row0 + rr < g.m)
                            *reinterpret_cast<uint4*>(dst_head + (long long)(row0 + rr) * rstride + c + q16 * 8) =
                                *reinterpret_cast<const uint4*>(stg + rr * STG_ROW + q16 * 16);
                    }
                    __syncwarp();
                };
                // RoPE on (a, b) with the table entries of channels d, d + 1
                auto rot2 = [&](int d, float& a0, float& b0, float& a1, float& b1) {
                    const int pr = (d / PAIR_SPAN) * HALF + (d & (HALF - 1));
                    const float4 cs = __ldg(reinterpret_cast<const float4*>(rt + pr));
                    float a = a0, b = b0;
                    a0 = a * cs.x - b * cs.y;
                    b0 = b * cs.x + a * cs.y;
                    a = a1;
                    b = b1;
                    a1 = a * cs.z - b * cs.w;
                    b1 = b * cs.z + a * cs.w;
                };
                if (QQ && part == 0) {
                    // Q also quantised here, as sp_prep's Q role would from the
                    // bf16 Q this epilogue writes (sage_quant.cu prep_q: one
                    // scale per 16 rows, 127 / amax, round to nearest even,
                    // clamp to +-127, q_scale = amax / 127 * q_mul).  The
                    // head's bf16 values stay in registers (packed) until the
                    // 16-row maximum is known; lanes 0-15 and 16-31 of a warp
                    // are two groups of consecutive rows.
                    uint32_t qp[D / 2];
                    float qmax = 0.f;
                    auto keep = [&](int c, const float (&x)[32]) {
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const uint32_t w = pack_bf16x2(x[e], x[e + 1]);
                            qp[(c + e) / 2] = w;
                            qmax = fmaxf(qmax, fmaxf(fabsf(__uint_as_float(w << 16)),
                                                     fabsf(__uint_as_float(w & 0xffff0000u))));
                        }
                    };
                    if (HALF >= 32) {
#pragma unroll
                        for (int c = 0; c < D; c += 32) {
                            if (c & HALF) continue;
                            float xa[32], xb[32];
                            load(c, xa);
                            load(c + HALF, xb);
#pragma unroll
                            for (int i = 0; i < 32; i += 2) rot2(c + i, xa[i], xb[i], xa[i + 1], xb[i + 1]);
                            if (q_out) {
                                store(c, xa);
                                store(c + HALF, xb);
                            }
                            keep(c, xa);
                            keep(c + HALF, xb);
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < D; c += 32) {
                            float xa[32];
                            load(c, xa);
                            if (HALF) {
#pragma unroll
                                for (int i = 0; i < HALF; i += 2)
                                    rot2(c + i, xa[i], xa[i + HALF], xa[i + 1], xa[i + HALF + 1]);
                            }
                            if (q_out) store(c, xa);
                            keep(c, xa);
                        }
                    }
#pragma unroll
                    for (int o = 1; o < 16; o <<= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, o));
                    const float inv = qmax > 0.f ? 127.0f / qmax : 0.f;
                    const bool fast = s8_fast(qmax);
                    if (row < g.m) {
                        const long long bhq = (long long)bb * g.hq + head;
                        int8_t* q8row = g.q8 + (bhq * g.tq_pad + tok) * D;
                        auto lo = [](uint32_t w) { return __uint_as_float(w << 16); };
                        auto hi = [](uint32_t w) { return __uint_as_float(w & 0xffff0000u); };
#pragma unroll
                        for (int i = 0; i < D / 16; i++) {
                            const uint32_t* p = qp + 8 * i;
                            const uint4 w = make_uint4(
                                s8x4(lo(p[0]) * inv, hi(p[0]) * inv, lo(p[1]) * inv, hi(p[1]) * inv, fast),
                                s8x4(lo(p[2]) * inv, hi(p[2]) * inv, lo(p[3]) * inv, hi(p[3]) * inv, fast),
                                s8x4(lo(p[4]) * inv, hi(p[4]) * inv, lo(p[5]) * inv, hi(p[5]) * inv, fast),
                                s8x4(lo(p[6]) * inv, hi(p[6]) * inv, lo(p[7]) * inv, hi(p[7]) * inv, fast));
                            *reinterpret_cast<uint4*>(q8row + 16 * i) = w;
                        }
                        if ((lane & 15) == 0)
                            g.q_scale[bhq * (g.tq_pad / QGROUP) + tok / QGROUP] = (qmax * (1.0f / 127.0f)) * g.q_mul;
                    }
                } else if (HALF >= 32) {
                    // chunk c and its partner chunk c + HALF
#pragma unroll 1
                    for (int c = 0; c < D; c += 32) {
                        if (c & HALF) continue;
                        float xa[32], xb[32];
                        load(c, xa);
                        load(c + HALF, xb);
                        if (part < 2) {
#pragma unroll
                            for (int i = 0; i < 32; i += 2) rot2(c + i, xa[i], xb[i], xa[i + 1], xb[i + 1]);
                        }
                        store(c, xa);
                        store(c + HALF, xb);
                    }
                } else {
                    // no RoPE, or pairs (d, d + 16) inside each 32-channel chunk
#pragma unroll 1
                    for (int c = 0; c < D; c += 32) {
                        float xa[32];
                        load(c, xa);
                        if (HALF && part < 2) {
#pragma unroll
                            for (int i = 0; i < HALF; i += 2) rot2(c + i, xa[i], xa[i + HALF], xa[i + 1], xa[i + HALF + 1]);
                        }
                        store(c, xa);
                    }
                }
            }
            // this CTA's rows of accumulator ab are read (this warp's half):
            // one arrival per warp on the leader's barrier
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_rank(bar(acc_empty[ab]), 0));
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader's MMAs have finished with both CTAs' memory
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, 2 * BN);
}

template <int D, int HALF, bool FP8, bool QQ, int EPW>
static cudaError_t qkv2_t(const QkvMaps& maps, const uint16_t* bias, const float* rope, const float* x_scale,
                          const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v, uint32_t* err,
                          const QkvGeom& g, cudaStream_t st) {
    auto kern = sp_qkv_gemm_2sm<D, HALF, FP8, QQ, EPW>;
    static std::atomic<unsigned> attr_set{0};  // one bit per device ordinal
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(attr_set.load(std::memory_order_acquire) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2::smem_bytes(EPW));
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
    const long long ntiles = (long long)(g.n / gemm2::BN) * ((g.m + 2 * gemm2::BM - 1) / (2 * gemm2::BM));
    long long pairs = n_sm / 2;
    if (ntiles < pairs) pairs = ntiles;
    if (pairs < 1) pairs = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(gemm2::nthreads(EPW));
    cfg.dynamicSmemBytes = gemm2::smem_bytes(EPW);
    cfg.stream = st;
    cudaLaunchAttribute attr[2] = {};
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // may start while the previous kernel on the stream finishes (griddep_wait
    // above keeps every memory access after that kernel's end)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, maps.x, maps.w, bias, (const float2*)rope, x_scale, w_scale, q, k, v, err, g);
}

template <bool FP8, bool QQ, int EPW>
static cudaError_t qkv2_dispatch_epw(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                     const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k,
                                     uint16_t* v, uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    const int half = rope ? g.rope_half : 0;
    if (d == 64) {
        if (half == 0) return qkv2_t<64, 0, FP8, QQ, EPW>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        if (half == 16) return qkv2_t<64, 16, FP8, QQ, EPW>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        if (half == 32) return qkv2_t<64, 32, FP8, QQ, EPW>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        return cudaErrorInvalidValue;
    }
    if constexpr (QQ && EPW == 8) {
        return cudaErrorInvalidValue;  // never chosen (epilogue_warps)
    } else {
        if (half == 0) return qkv2_t<128, 0, FP8, QQ, EPW>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        if (half == 64)
            return qkv2_t<128, 64, FP8, QQ, EPW>(maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        return cudaErrorInvalidValue;
    }
}

template <bool FP8, bool QQ>
static cudaError_t qkv2_dispatch(int d, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                 const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                 uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    if constexpr (FP8) {
        return qkv2_dispatch_epw<FP8, QQ, 8>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
    } else {
        if (gemm2::epilogue_warps(FP8, QQ, d, g.k) == 8)
            return qkv2_dispatch_epw<FP8, QQ, 8>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
        return qkv2_dispatch_epw<FP8, QQ, 4>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
    }
}

cudaError_t launch_qkv_gemm_2sm(int d, bool fp8, const QkvMaps& maps, const uint16_t* bias, const float* rope,
                                const float* x_scale, const float* w_scale, uint16_t* q, uint16_t* k, uint16_t* v,
                                uint32_t* err, const QkvGeom& g, cudaStream_t st) {
    if (fp8) return qkv2_dispatch<true, false>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
    // bf16: with g.q8 set, Q is quantised in the epilogue (q may then be null)
    return g.q8 ? qkv2_dispatch<false, true>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st)
                : qkv2_dispatch<false, false>(d, maps, bias, rope, x_scale, w_scale, q, k, v, err, g, st);
}

}  // namespace sp
