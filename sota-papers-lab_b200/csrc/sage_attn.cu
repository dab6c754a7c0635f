// SageAttention2 attention for sm_100a on the 5th-generation tensor cores.
//
// Math (the reference kernel's, platform/spl-nn/cuda/sage_attn.cu:1-20,
// 227-344): S = Q8 K8^T in INT8 -> S32; x = S * q_scale * k_scale (+ log2
// count bias when keys are merged), q_scale already holding softmax scale *
// log2(e); online softmax in exp2 with a running max m and sum l;
// P = 448 * 2^(x - m) rounded to FP8 E4M3; each block's PV starts from zero
// (FP32) and is folded into the FP32 output O = O * alpha + PV (two-level
// accumulation); out = O / l * v_scale + v_mean in bf16.  The S accumulator
// is read as the float 1.5 * 2^23 + S (exact for |S| < 2^22) after one
// integer add, and the 1.5 * 2^23 offset is folded into the exp2 FFMA, as
// the reference does.
//
// Structure (one CTA = 128 query rows of one (batch, q head); 12 warps):
//   warp 0     TMA producer: Q once, then a ring of 128-key INT8 K tiles and
//              a ring of [D][128] FP8 V^T tiles (non-multicast TMA, 128B or
//              64B swizzle, zero fill past the end)
//   warp 1     MMA issuer (one thread): QK^T = tcgen05.mma kind::i8 M128 N128
//              into a double-buffered S in TMEM; PV = tcgen05.mma
//              kind::f8f6f4 M128 N=D with P from shared memory into a PV
//              buffer in TMEM
//   warp 2     TMEM allocation (512 columns)
//   warps 4-7  softmax: thread = query row (TMEM lane), reads its S row with
//              tcgen05.ld, computes m, alpha, P8 and l in registers, writes
//              its P row into the 128B-swizzled K-major P tile
//   warps 8-11 correction: O (FP32, TMEM) = O * alpha + PV per block, then
//              the epilogue
// Extensions not in the reference: causal masking (blocks past the diagonal
// are skipped, the diagonal block masked) and GQA (q head h reads kv head
// h / (heads / kv_heads)).
//
// Every mbarrier wait is bounded (sage_dev.cuh): on a timeout the kernel
// records it in the device error word, drains its own TMA loads and MMAs,
// frees TMEM and returns.
#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

constexpr int KST = 3;   // K ring depth
constexpr int VST = 3;   // V ring depth
constexpr int NTHREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t MAGIC_I = 0x4B400000u;    // bits of 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;       // 1.5 * 2^23
constexpr float LOG2_448 = 8.807354922057604f;

template <int D>
struct AttnSmem {
    static constexpr int Q_BYTES = 128 * D;
    static constexpr int K_BYTES = 128 * D;
    static constexpr int V_BYTES = D * 128;
    static constexpr int P_BYTES = 128 * 128;
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + Q_BYTES;
    static constexpr int V_OFF = K_OFF + KST * K_BYTES;
    static constexpr int P_OFF = V_OFF + VST * V_BYTES;
    static constexpr int END = P_OFF + 2 * P_BYTES;
    static constexpr int DYN = END + 1024;  // slack to align the base to 1024
};

struct Bars {
    uint64_t q_full;
    uint64_t k_full[KST], k_empty[KST];
    uint64_t v_full[VST], v_empty[VST];
    uint64_t s_full[2];
    uint64_t p_full[2], p_free[2];
    uint64_t pv_full, pv_free;
    uint64_t a_full[2], a_free[2];
    uint64_t l_full;
    uint64_t mma_done;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// All 32 lanes wait; the warp gives up together if any lane gave up.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint32_t* err, uint32_t site) {
    const bool ok = mbar_wait(bar, parity, err, site);
    return __all_sync(0xffffffffu, ok);
}

template <int D, bool CAUSAL, bool MERGE>
__global__ void __launch_bounds__(NTHREADS, 1)
    sp_attn(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
            const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q_scale,
            const float* __restrict__ k_scale, const float* __restrict__ stats, const float* __restrict__ kbias,
            uint16_t* __restrict__ out, uint32_t* __restrict__ err, const Geom g) {
    using L = AttnSmem<D>;
    constexpr uint32_t SWZ = D == 128 ? SWZ_128B : SWZ_64B;
    constexpr uint32_t QK_SBO = 8 * D;  // 8 rows of D bytes
    constexpr uint32_t IDESC_QK = make_idesc(C_S32, F_S8, F_S8, 128, 128);
    constexpr uint32_t IDESC_PV = make_idesc(C_F32, F_E4M3, F_E4M3, 128, D);
    constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_PV = 256, TM_O = 256 + (D == 128 ? 128 : 64);

    extern __shared__ uint8_t dyn_smem[];
    __shared__ Bars bars;
    __shared__ uint32_t tmem_base_s;
    __shared__ uint32_t abort_s;
    __shared__ float alpha_s[2][128];
    __shared__ float l_s[128];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh_q = blockIdx.x;
    const int n_qt = g.tq_pad / 128;
    const int qt = CAUSAL ? n_qt - 1 - (int)blockIdx.y : (int)blockIdx.y;
    const int b = bh_q / g.heads, h = bh_q % g.heads;
    const int group = g.heads / g.kv_heads;
    const int bh_kv = b * g.kv_heads + h / group;
    const int nkb64 = g.tk_pad / KBLOCK;
    const int nkb = (g.tk + BLK - 1) / BLK;
    const int nb = CAUSAL ? min(nkb, qt + 1) : nkb;

    const uint32_t sbase = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const uint32_t sQ = sbase + L::Q_OFF, sK = sbase + L::K_OFF, sV = sbase + L::V_OFF, sP = sbase + L::P_OFF;
    auto bar = [](uint64_t& x) { return smem_u32(&x); };

    if (tid == 0) {
        abort_s = ld_volatile(err) != 0 ? 1u : 0u;
        mbar_init(bar(bars.q_full), 1);
        for (int i = 0; i < KST; i++) {
            mbar_init(bar(bars.k_full[i]), 1);
            mbar_init(bar(bars.k_empty[i]), 1);
        }
        for (int i = 0; i < VST; i++) {
            mbar_init(bar(bars.v_full[i]), 1);
            mbar_init(bar(bars.v_empty[i]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(bars.s_full[i]), 1);
            mbar_init(bar(bars.p_full[i]), 128);
            mbar_init(bar(bars.p_free[i]), 1);
            mbar_init(bar(bars.a_full[i]), 128);
            mbar_init(bar(bars.a_free[i]), 128);
        }
        mbar_init(bar(bars.pv_full), 1);
        mbar_init(bar(bars.pv_free), 128);
        mbar_init(bar(bars.l_full), 128);
        mbar_init(bar(bars.mma_done), 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (abort_s) return;  // uniform: an earlier CTA already failed
    if (warp == 2) {
        tmem_alloc(smem_u32(&tmem_base_s), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&map_q);
            tma_prefetch_desc(&map_k);
            tma_prefetch_desc(&map_v);
            mbar_expect_tx(bar(bars.q_full), L::Q_BYTES);
            tma_load_3d(sQ, &map_q, bar(bars.q_full), 0, qt * 128, bh_q);
            int nk = 0, nv = 0;
            for (int j = 0; j < nb; j++) {
                const int ks = j % KST, vs = j % VST;
                if (j >= KST && !mbar_wait(bar(bars.k_empty[ks]), ((j / KST) - 1) & 1, err, 1)) break;
                mbar_expect_tx(bar(bars.k_full[ks]), L::K_BYTES);
                tma_load_3d(sK + ks * L::K_BYTES, &map_k, bar(bars.k_full[ks]), 0, j * BLK, bh_kv);
                nk++;
                if (j >= VST && !mbar_wait(bar(bars.v_empty[vs]), ((j / VST) - 1) & 1, err, 2)) break;
                mbar_expect_tx(bar(bars.v_full[vs]), L::V_BYTES);
                tma_load_3d(sV + vs * L::V_BYTES, &map_v, bar(bars.v_full[vs]), j * BLK, 0, bh_kv);
                nv++;
            }
            // Drain: every load issued lands before the CTA exits (these
            // waits ignore the error word and stop only at the time limit).
            mbar_wait(bar(bars.q_full), 0, err, 3, false);
            for (int s = 0; s < KST && s < nk; s++) {
                const int last = s + ((nk - 1 - s) / KST) * KST;
                mbar_wait(bar(bars.k_full[s]), (last / KST) & 1, err, 4, false);
            }
            for (int s = 0; s < VST && s < nv; s++) {
                const int last = s + ((nv - 1 - s) / VST) * VST;
                mbar_wait(bar(bars.v_full[s]), (last / VST) & 1, err, 5, false);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            bool ok = mbar_wait(bar(bars.q_full), 0, err, 10);
            auto issue_qk = [&](int jj) -> bool {
                const int s = jj % KST;
                if (!mbar_wait(bar(bars.k_full[s]), (jj / KST) & 1, err, 11)) return false;
                tc_fence_after();
                const uint32_t d_s = tmem + ((jj & 1) ? TM_S1 : TM_S0);
                const uint32_t kaddr = sK + s * L::K_BYTES;
#pragma unroll
                for (int kk = 0; kk < D / 32; kk++)
                    umma_i8(d_s, smem_desc(sQ + kk * 32, QK_SBO, SWZ), smem_desc(kaddr + kk * 32, QK_SBO, SWZ),
                            IDESC_QK, kk > 0);
                tc_commit(bar(bars.s_full[jj & 1]));
                tc_commit(bar(bars.k_empty[s]));
                return true;
            };
            if (ok) ok = issue_qk(0);
            if (ok && nb > 1) ok = issue_qk(1);
            for (int j = 0; j < nb && ok; j++) {
                const int pb = j & 1, vs = j % VST;
                ok = mbar_wait(bar(bars.p_full[pb]), (j >> 1) & 1, err, 12);
                if (ok && j >= 1) ok = mbar_wait(bar(bars.pv_free), (j - 1) & 1, err, 13);
                if (ok) ok = mbar_wait(bar(bars.v_full[vs]), (j / VST) & 1, err, 14);
                if (!ok) break;
                tc_fence_after();
                const uint32_t paddr = sP + pb * L::P_BYTES, vaddr = sV + vs * L::V_BYTES;
#pragma unroll
                for (int kk = 0; kk < BLK / 32; kk++)
                    umma_f8(tmem + TM_PV, smem_desc(paddr + kk * 32, 1024, SWZ_128B),
                            smem_desc(vaddr + kk * 32, 1024, SWZ_128B), IDESC_PV, kk > 0);
                tc_commit(bar(bars.pv_full));
                tc_commit(bar(bars.v_empty[vs]));
                tc_commit(bar(bars.p_free[pb]));
                if (j + 2 < nb) ok = issue_qk(j + 2);
            }
            // No MMA may be in flight when TMEM is freed.
            tc_commit(bar(bars.mma_done));
            mbar_wait(bar(bars.mma_done), 0, err, 15, false);
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ softmax
        const int r = tid - 128;                       // query row in the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)((warp - 4) * 32) << 16;
        const int qrow = qt * 128 + r;
        const float qs = q_scale[(long long)bh_q * (g.tq_pad / QGROUP) + qrow / QGROUP];
        const float* ksc = k_scale + (long long)bh_kv * nkb64;
        float m = -1.0e30f, l = 0.f;
        const uint32_t prow = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
        bool ok = true;
        for (int j = 0; j < nb; j++) {
            const int sb = j & 1;
            const float ks0 = ksc[2 * j];
            const float ks1 = (2 * j + 1 < nkb64) ? ksc[2 * j + 1] : ks0;
            const float sc0 = qs * ks0, sc1 = qs * ks1;
            if (!warp_wait(bar(bars.s_full[sb]), (j >> 1) & 1, err, 20)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[128];
            {
                uint32_t (&c0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[0]);
                uint32_t (&c1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32]);
                uint32_t (&c2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[64]);
                uint32_t (&c3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[96]);
                const uint32_t ts = tmem + lane_off + (sb ? TM_S1 : TM_S0);
                tmem_ld32(ts + 0, c0);
                tmem_ld32(ts + 32, c1);
                tmem_ld32(ts + 64, c2);
                tmem_ld32(ts + 96, c3);
                tmem_wait_ld();
            }
            // x: the float 1.5 * 2^23 + S, or the log2 logit when merging;
            // masked keys -inf.
            float x[128];
            const int key0 = j * BLK;
            const bool tail = key0 + BLK > g.tk;
            const bool diag = CAUSAL && (key0 + BLK > qt * 128);
            if (MERGE) {
                const float c0 = -MAGIC_F * sc0, c1 = -MAGIC_F * sc1;
#pragma unroll
                for (int c = 0; c < 128; c++) {
                    const int key = key0 + c;
                    const float kb = key < g.tk_pad ? __ldg(kbias + key) : __int_as_float(0xff800000);
                    x[c] = fmaf(__uint_as_float(sr[c] + MAGIC_I), c < 64 ? sc0 : sc1, kb + (c < 64 ? c0 : c1));
                }
            } else {
#pragma unroll
                for (int c = 0; c < 128; c++) x[c] = __uint_as_float(sr[c] + MAGIC_I);
            }
            if (tail || diag) {
#pragma unroll
                for (int c = 0; c < 128; c++) {
                    const int key = key0 + c;
                    if (key >= g.tk || (CAUSAL && key > qrow)) x[c] = __int_as_float(0xff800000);
                }
            }
            float mnew;
            if (MERGE) {
                float mx = x[0];
#pragma unroll
                for (int c = 1; c < 127; c += 2) mx = fmax3(mx, x[c], x[c + 1]);
                mx = fmaxf(mx, x[127]);
                mnew = fmaxf(m, mx);
            } else {
                float m0 = x[0], m1 = x[64];
#pragma unroll
                for (int c = 1; c < 63; c += 2) {
                    m0 = fmax3(m0, x[c], x[c + 1]);
                    m1 = fmax3(m1, x[64 + c], x[64 + c + 1]);
                }
                m0 = fmaxf(m0, x[63]);
                m1 = fmaxf(m1, x[127]);
                mnew = fmax3(m, fmaf(m0, sc0, -MAGIC_F * sc0), fmaf(m1, sc1, -MAGIC_F * sc1));
            }
            const float alpha = ex2(m - mnew);
            m = mnew;
            // P = 448 * 2^(x - m) as E4M3, written to the swizzled P tile.
            if (j >= 2 && !warp_wait(bar(bars.p_free[sb]), ((j >> 1) - 1) & 1, err, 21)) {
                ok = false;
                break;
            }
            const uint32_t prow_addr = sP + sb * L::P_BYTES + prow;
            float sum = 0.f;
#pragma unroll
            for (int c16 = 0; c16 < 8; c16++) {
                float p[16];
                const float sc = c16 < 4 ? sc0 : sc1;
                const float off = MERGE ? LOG2_448 - mnew : LOG2_448 - mnew - MAGIC_F * sc;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const float y = x[c16 * 16 + e];
                    p[e] = ex2(MERGE ? y + off : fmaf(y, sc, off));
                    sum += p[e];
                }
                uint32_t w[4];
#pragma unroll
                for (int q4 = 0; q4 < 4; q4++)
                    w[q4] = e4m3x2(p[4 * q4], p[4 * q4 + 1]) | (e4m3x2(p[4 * q4 + 2], p[4 * q4 + 3]) << 16);
                const uint32_t a = prow_addr + (uint32_t)(((c16 ^ (r & 7)) & 7) << 4);
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                             "r"(w[3])
                             : "memory");
            }
            l = fmaf(l, alpha, sum);
            fence_proxy_async_smem();
            tc_fence_before();
            if (j >= 2 && !warp_wait(bar(bars.a_free[sb]), ((j >> 1) - 1) & 1, err, 22)) {
                ok = false;
                break;
            }
            alpha_s[sb][r] = alpha;
            mbar_arrive(bar(bars.a_full[sb]));
            mbar_arrive(bar(bars.p_full[sb]));
        }
        if (ok) {
            l_s[r] = l;
            mbar_arrive(bar(bars.l_full));
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ correction + epilogue
        const int r = tid - 256;
        const uint32_t lane_off = (uint32_t)((warp - 8) * 32) << 16;
        const uint32_t t_pv = tmem + lane_off + TM_PV, t_o = tmem + lane_off + TM_O;
        bool ok = true;
        for (int j = 0; j < nb; j++) {
            const int sb = j & 1;
            if (!warp_wait(bar(bars.a_full[sb]), (j >> 1) & 1, err, 30)) {
                ok = false;
                break;
            }
            const float alpha = alpha_s[sb][r];
            mbar_arrive(bar(bars.a_free[sb]));
            if (!warp_wait(bar(bars.pv_full), j & 1, err, 31)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                uint32_t pv[32], o[32];
                tmem_ld32(t_pv + c * 32, pv);
                if (j > 0) {
                    tmem_ld32(t_o + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++)
                        o[e] = __float_as_uint(fmaf(__uint_as_float(o[e]), alpha, __uint_as_float(pv[e])));
                    tmem_st32(t_o + c * 32, o);
                } else {
                    tmem_wait_ld();
                    tmem_st32(t_o + c * 32, pv);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(bars.pv_free));
        }
        if (ok && warp_wait(bar(bars.l_full), 0, err, 32)) {
            tc_fence_after();
            const float inv = 1.0f / l_s[r];
            const int row = qt * 128 + r;
            const float* vmean = stats + (long long)bh_kv * 4 * D + D;
            const float* vscale = vmean + D;
            uint16_t* orow = out + (long long)b * g.o_sb + (long long)row * g.o_st + (long long)h * g.o_sh;
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                uint32_t o[32];
                tmem_ld32(t_o + c * 32, o);
                tmem_wait_ld();
                if (row < g.tokens) {
#pragma unroll
                    for (int e8 = 0; e8 < 4; e8++) {
                        uint32_t w[4];
#pragma unroll
                        for (int e2 = 0; e2 < 4; e2++) {
                            const int e = e8 * 8 + e2 * 2, d = c * 32 + e;
                            const float y0 = fmaf(__uint_as_float(o[e]) * inv, __ldg(vscale + d), __ldg(vmean + d));
                            const float y1 =
                                fmaf(__uint_as_float(o[e + 1]) * inv, __ldg(vscale + d + 1), __ldg(vmean + d + 1));
                            w[e2] = pack_bf16x2(y0, y1);
                        }
                        *reinterpret_cast<uint4*>(orow + c * 32 + e8 * 8) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, TMEM_COLS);
}

template <int D, bool CAUSAL, bool MERGE>
static cudaError_t attend_t(const AttnMaps& maps, const Buffers& buf, const Geom& g, void* out, cudaStream_t st) {
    static unsigned attr_set = 0;  // one bit per device ordinal
    auto kern = sp_attn<D, CAUSAL, MERGE>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(attr_set & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem<D>::DYN);
        if (e != cudaSuccess) return e;
        if (dev < 32) attr_set |= 1u << dev;
    }
    dim3 grid(g.batch * g.heads, g.tq_pad / 128);
    kern<<<grid, NTHREADS, AttnSmem<D>::DYN, st>>>(maps.q, maps.k, maps.v, buf.q_scale, buf.k_scale, buf.stats,
                                                   buf.kbias, (uint16_t*)out, buf.err, g);
    return cudaGetLastError();
}

cudaError_t launch_attend(int d, const AttnMaps& maps, const Buffers& buf, const Geom& g, void* out,
                          cudaStream_t st) {
    const bool merge = g.merge > 1, causal = g.causal != 0;
    if (d == 64) {
        if (merge) return attend_t<64, false, true>(maps, buf, g, out, st);
        return causal ? attend_t<64, true, false>(maps, buf, g, out, st)
                      : attend_t<64, false, false>(maps, buf, g, out, st);
    }
    if (merge) return attend_t<128, false, true>(maps, buf, g, out, st);
    return causal ? attend_t<128, true, false>(maps, buf, g, out, st)
                  : attend_t<128, false, false>(maps, buf, g, out, st);
}

cudaError_t attn_func_attributes(int d, int merge, int* regs, int* local_bytes) {
    cudaFuncAttributes a;
    cudaError_t e = d == 64 ? (merge ? cudaFuncGetAttributes(&a, sp_attn<64, false, true>)
                                     : cudaFuncGetAttributes(&a, sp_attn<64, false, false>))
                            : (merge ? cudaFuncGetAttributes(&a, sp_attn<128, false, true>)
                                     : cudaFuncGetAttributes(&a, sp_attn<128, false, false>));
    if (e != cudaSuccess) return e;
    *regs = a.numRegs;
    *local_bytes = (int)a.localSizeBytes;
    return cudaSuccess;
}

int attn_smem_bytes(int d) { return d == 64 ? AttnSmem<64>::DYN : AttnSmem<128>::DYN; }

}  // namespace sp
