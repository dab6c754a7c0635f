// SageAttention2 attention for sm_100a on the 5th-generation tensor cores.
//
// Math (the reference kernel's, platform/spl-nn/cuda/sage_attn.cu:1-20,
// 227-344): S = Q8 K8^T in INT8 -> S32; x = S * q_scale * k_scale (+ log2
// count bias when keys are merged), q_scale already holding softmax scale *
// log2(e); online softmax in exp2 with a running max m and sum l;
// P = 448 * 2^(x - m) rounded to FP8 E4M3; each block's PV starts from zero
// (FP32, in TMEM) and is folded into the FP32 output O = O * alpha + PV held
// in registers (two-level accumulation); out = O / l * v_scale + v_mean in
// bf16.  The S accumulator starts at the integer 1.5 * 2^23 (copied from
// shared memory by tcgen05.cp ahead of each QK^T), so the finished S32 value
// read as a float is 1.5 * 2^23 + S (exact for |S| < 2^22); the offset folds
// into the exp2 FFMA, as the reference's float trick does.
//
// Structure: persistent, one CTA per SM working through 128-row query tiles
// of (batch, q head) in turn (causal: the heaviest first); every ring and
// buffer carries on from one tile to the next, so a tile's output is written
// while the next tile's loads and QK^T run.  12 warps.
//   warps 0-7  softmax + correction.  Warp w owns the 16 rows
//              32*(w%4) + 16*(w/4) + (0..15) (its TMEM lane quarter is w%4);
//              lane t < 16 handles keys 0-63 of every 128-key block and
//              output columns [0, D/2) of row t, lane t + 16 keys 64-127
//              and columns [D/2, D) of the same row.  S is read with
//              tcgen05.ld 16x32bx2, so the two halves of a row meet in one
//              warp (one shuffle for the row max) and the two warps sharing
//              an SM sub-partition run independently.  Keys 0-63 and 64-127
//              are two 64-key k_scale blocks, so each lane has one scale.
//   warps 8-11 one service thread each, one per SM sub-partition (issuing
//              TMA and tcgen05.mma costs the issuing sub-partition cycles):
//              8: Q once and a ring of 128-key INT8 K tiles, 9: a ring of
//              [D][128] FP8 V^T tiles (non-multicast TMA, 128B / 64B swizzle,
//              zero fill past the end); 10: TMEM allocation and QK^T =
//              tcgen05.mma kind::i8 M128 N128 into a double-buffered S;
//              11: PV = tcgen05.mma kind::f8f6f4 M128 N=D with P from shared
//              memory into a double-buffered PV
// Per 16 keys, exp_poly<D>() of the exponentials run on the FMA pipe
// (exp2_poly2) to take load off the MUFU unit.
// Extensions not in the reference: causal masking (blocks past the diagonal
// are skipped, the diagonal block masked) and GQA (q head h reads kv head
// h / (heads / kv_heads)).
//
// Every mbarrier wait is bounded (sage_dev.cuh): on a timeout the kernel
// records it in the device error word, drains its own TMA loads and MMAs,
// frees TMEM and returns.
#include <atomic>

#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

constexpr int KST = 3;   // K ring depth
constexpr int VST = 3;   // V ring depth
// Of every 16 exponentials, how many run on the FMA pipe (exp2_poly2): 4 at
// D = 128, 6 at D = 64, whose PV fold leaves the FMA pipe more room
// (measured: C4 2.052 ms with 4 against 2.108 with 6; C2 0.1235 ms with 6
// against 0.1271 with 4).
#ifndef SP_EXP_POLY_128
#define SP_EXP_POLY_128 4
#endif
#ifndef SP_EXP_POLY_64
#define SP_EXP_POLY_64 6
#endif
template <int D>
constexpr int exp_poly() { return D == 64 ? SP_EXP_POLY_64 : SP_EXP_POLY_128; }
constexpr int NTHREADS = 384;
// One service thread per SM sub-partition (warp % 4), so that no pair of
// softmax warps carries more issue load than another: K loads (and Q),
// V loads, the QK^T MMAs, the PV MMAs.
constexpr int K_WARP = 8, V_WARP = 9, QK_WARP = 10, PV_WARP = 11, NSOFTMAX_WARPS = 8;
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
    static constexpr int K_OFF = Q_OFF + 2 * Q_BYTES;  // Q double-buffered (consecutive tiles)
    static constexpr int V_OFF = K_OFF + KST * K_BYTES;
    static constexpr int P_OFF = V_OFF + VST * V_BYTES;
    static constexpr int M_OFF = P_OFF + 2 * P_BYTES;  // 4 KB of 1.5 * 2^23 for the S refill
    // (D = 64) each softmax warp's 16 output rows (bf16), padded by 16 bytes
    // per row, so that the epilogue's global stores cover whole rows
    static constexpr int STAGE_ROW = 2 * D + 16;
    static constexpr int STAGE_OFF = M_OFF + 4096;
    static constexpr int END = STAGE_OFF + (D == 64 ? NSOFTMAX_WARPS * 16 * STAGE_ROW : 0);
    static constexpr int DYN = END + 1024;  // slack to align the base to 1024
};

struct Bars {
    uint64_t q_full[2], q_empty[2];
    uint64_t k_full[KST], k_empty[KST];
    uint64_t v_full[VST], v_empty[VST];
    uint64_t s_full[2];
    uint64_t p_full[2], p_free[2];
    uint64_t qk_done, pv_done;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint32_t* err, uint32_t site) {
    return warp_all_wait(bar, parity, err, site);
}

// PARTIAL (context parallelism): query tile i of the segment is tile
// q_tile0 + i of the workspace, the keys are keys k_key0 .. k_key0 + tk of
// the K/V buffer (CAUSAL then means key i is seen by query i and later of
// the segment); the result is merged into the fp32 accumulator acc and the
// per-row log2 softmax denominator lse by log-sum-exp instead of written.
// GQ (causal, not PARTIAL): the queries are two chunks of a longer
// sequence whose keys are all gathered (g.q_split, g.q_goff0, g.q_goff1).
template <int D, bool CAUSAL, bool MERGE, bool PARTIAL, bool GQ = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    sp_attn(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
            const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q_scale,
            const float* __restrict__ k_scale, const float* __restrict__ stats, const float* __restrict__ kbias,
            uint16_t* __restrict__ out, float* __restrict__ acc, float* __restrict__ lse, uint32_t* __restrict__ err,
            const Geom g) {
    using L = AttnSmem<D>;
    constexpr int DH = D / 2;
    constexpr uint32_t SWZ = D == 128 ? SWZ_128B : SWZ_64B;
    constexpr uint32_t QK_SBO = 8 * D;  // 8 rows of D bytes
    constexpr uint32_t IDESC_QK = make_idesc(C_S32, F_S8, F_S8, 128, 128);
    constexpr uint32_t IDESC_PV = make_idesc(C_F32, F_E4M3, F_E4M3, 128, D);
    constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_PV0 = 256, TM_PV1 = 256 + D;

    extern __shared__ uint8_t dyn_smem[];
    __shared__ Bars bars;
    __shared__ uint32_t tmem_base_s;
    __shared__ uint32_t abort_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Persistent: each CTA takes one tile of every round of gridDim.x tiles
    // (tile_at).  Tile t is query tile row t / (B*H) (causal: the heaviest
    // rows first) of (batch, head) t % (B*H), so that CTAs running together
    // share each kv head's K/V.
    const int n_qt = g.q_tiles;  // query tiles per (batch, head) (of the segment)
    const int n_bh = g.batch * g.heads;
    const int ntiles = n_bh * n_qt;
    const int group = g.heads / g.kv_heads;
    const int nkb64 = g.tk_pad / KBLOCK;  // k_scale row length of the K/V buffer
    // segment offsets (context parallelism only; compile-time zero otherwise)
    const int q_tile0 = PARTIAL ? g.q_tile0 : 0, k_key0 = PARTIAL ? g.k_key0 : 0;
    const int nkb64_seg = PARTIAL ? (g.tk + KBLOCK - 1) / KBLOCK : nkb64;  // 64-key blocks attended
    const int nkb = (g.tk + BLK - 1) / BLK;
    // The CTA's it-th tile: round it of gridDim.x tiles, taken forwards in
    // even rounds and backwards in odd ones, so that the heavy causal tiles
    // of one round and the light ones of the next share a CTA.
    auto tile_at = [&](int it) {
        const int c = (it & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
        return it * (int)gridDim.x + c;
    };
    struct Tile {
        int bh_q, b, h, bh_kv, qt, nb, g0;
    };
    auto tile_of = [&](int t) {
        Tile x;
        const int qi = t / n_bh;
        x.bh_q = t % n_bh;
        x.b = x.bh_q / g.heads;
        x.h = x.bh_q % g.heads;
        x.bh_kv = x.b * g.kv_heads + x.h / group;
        x.qt = CAUSAL ? n_qt - 1 - qi : qi;  // tile within the segment
        // key position of the tile's first query row (causal over gathered
        // keys: its global row; otherwise its row in the segment)
        const int r0 = x.qt * 128;
        x.g0 = GQ ? (r0 < g.q_split ? g.q_goff0 + r0 : g.q_goff1 + (r0 - g.q_split)) : r0;
        x.nb = CAUSAL ? min(nkb, x.g0 / BLK + 1) : nkb;
        return x;
    };

    const uint32_t sbase = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const uint32_t sQ = sbase + L::Q_OFF, sK = sbase + L::K_OFF, sV = sbase + L::V_OFF, sP = sbase + L::P_OFF;
    const uint32_t sM = sbase + L::M_OFF;
    auto bar = [](uint64_t& x) { return smem_u32(&x); };

    for (int i = tid; i < 1024; i += NTHREADS)
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(sM + 4 * i), "r"(MAGIC_I) : "memory");
    fence_proxy_async_smem();
    if (tid == 0) {
        abort_s = ld_volatile(err) != 0 ? 1u : 0u;
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(bars.q_full[i]), 1);
            mbar_init(bar(bars.q_empty[i]), 1);
        }
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
            mbar_init(bar(bars.p_full[i]), NSOFTMAX_WARPS);
            mbar_init(bar(bars.p_free[i]), 1);
        }
        mbar_init(bar(bars.qk_done), 1);
        mbar_init(bar(bars.pv_done), 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (abort_s) return;  // uniform: an earlier CTA already failed
    if (warp == QK_WARP) {
        tmem_alloc(smem_u32(&tmem_base_s), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    // the set-up above may overlap the end of the quantiser launched before
    // this kernel; everything below reads what it wrote
    griddep_wait();

    // Every role walks the same tiles; J counts this CTA's 128-key blocks over
    // all its tiles and drives every ring index and phase, so the buffers
    // carry from one tile to the next.
    if (warp == K_WARP) {
        // ------------------------------------------------------------ Q and K loads
        if (lane == 0) {
            tma_prefetch_desc(&map_q);
            tma_prefetch_desc(&map_k);
            int J = 0, nq = 0;
            bool ok = true;
            for (int it = 0, t = tile_at(0); t < ntiles && ok; t = tile_at(++it)) {
                const Tile x = tile_of(t);
                const int qb = it & 1;
                // Q buffer qb is free once the QK^T of tile it - 2 is done
                if (it >= 2 && !mbar_wait(bar(bars.q_empty[qb]), ((it >> 1) - 1) & 1, err, 6)) break;
                mbar_expect_tx(bar(bars.q_full[qb]), L::Q_BYTES);
                tma_load_3d(sQ + qb * L::Q_BYTES, &map_q, bar(bars.q_full[qb]), 0, (q_tile0 + x.qt) * 128, x.bh_q);
                nq++;
                for (int j = 0; j < x.nb; j++) {
                    const int ks = J % KST;
                    if (J >= KST && !mbar_wait(bar(bars.k_empty[ks]), ((J / KST) - 1) & 1, err, 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(bar(bars.k_full[ks]), L::K_BYTES);
                    tma_load_3d(sK + ks * L::K_BYTES, &map_k, bar(bars.k_full[ks]), 0, k_key0 + j * BLK, x.bh_kv);
                    J++;
                }
            }
            // Drain: every load issued lands before the CTA exits (these
            // waits ignore the error word and stop only at the time limit).
            for (int qb = 0; qb < 2 && qb < nq; qb++) {
                const int last = qb + ((nq - 1 - qb) / 2) * 2;
                mbar_wait(bar(bars.q_full[qb]), (last >> 1) & 1, err, 3, false);
            }
            for (int s = 0; s < KST && s < J; s++) {
                const int last = s + ((J - 1 - s) / KST) * KST;
                mbar_wait(bar(bars.k_full[s]), (last / KST) & 1, err, 4, false);
            }
        }
    } else if (warp == V_WARP) {
        // ------------------------------------------------------------ V loads
        if (lane == 0) {
            tma_prefetch_desc(&map_v);
            int J = 0;
            bool ok = true;
            for (int it = 0, t = tile_at(0); t < ntiles && ok; t = tile_at(++it)) {
                const Tile x = tile_of(t);
                for (int j = 0; j < x.nb; j++) {
                    const int vs = J % VST;
                    if (J >= VST && !mbar_wait(bar(bars.v_empty[vs]), ((J / VST) - 1) & 1, err, 2)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(bar(bars.v_full[vs]), L::V_BYTES);
                    tma_load_3d(sV + vs * L::V_BYTES, &map_v, bar(bars.v_full[vs]), k_key0 + j * BLK, 0, x.bh_kv);
                    J++;
                }
            }
            for (int s = 0; s < VST && s < J; s++) {
                const int last = s + ((J - 1 - s) / VST) * VST;
                mbar_wait(bar(bars.v_full[s]), (last / VST) & 1, err, 5, false);
            }
        }
    } else if (warp == QK_WARP) {
        // ------------------------------------------------------------ QK^T issuer
        if (lane == 0) {
            const uint64_t mdesc = smem_desc(sM, 256, 0);  // 4 KB of 1.5 * 2^23 (no swizzle)
            int J = 0;
            bool ok = true;
            for (int it = 0, t = tile_at(0); t < ntiles && ok; t = tile_at(++it)) {
                const Tile x = tile_of(t);
                const int qb = it & 1;
                const uint32_t qaddr = sQ + qb * L::Q_BYTES;
                if (!(ok = mbar_wait(bar(bars.q_full[qb]), (it >> 1) & 1, err, 10))) break;
                for (int j = 0; j < x.nb; j++, J++) {
                    // S[J % 2] was read by every softmax warp (block J - 2)
                    if (J >= 2 && !(ok = mbar_wait(bar(bars.p_full[J & 1]), ((J - 2) >> 1) & 1, err, 12))) break;
                    const int s = J % KST;
                    if (!(ok = mbar_wait(bar(bars.k_full[s]), (J / KST) & 1, err, 11))) break;
                    tc_fence_after();
                    const uint32_t d_s = tmem + ((J & 1) ? TM_S1 : TM_S0);
                    const uint32_t kaddr = sK + s * L::K_BYTES;
                    // S starts at 1.5 * 2^23 (tcgen05.cp from shared memory, in
                    // issue order before the MMAs that accumulate onto it)
#pragma unroll
                    for (int c = 0; c < 128; c += 8) tmem_cp_128x256b(d_s + c, mdesc);
#pragma unroll
                    for (int kk = 0; kk < D / 32; kk++)
                        umma_i8(d_s, smem_desc(qaddr + kk * 32, QK_SBO, SWZ), smem_desc(kaddr + kk * 32, QK_SBO, SWZ),
                                IDESC_QK, 1);  // onto 1.5 * 2^23
                    tc_commit(bar(bars.s_full[J & 1]));
                    tc_commit(bar(bars.k_empty[s]));
                }
                if (ok) tc_commit(bar(bars.q_empty[qb]));  // the tile's Q is read once its MMAs complete
            }
            // No MMA may be in flight when TMEM is freed.
            tc_commit(bar(bars.qk_done));
            mbar_wait(bar(bars.qk_done), 0, err, 15, false);
        }
    } else if (warp == PV_WARP) {
        // ------------------------------------------------------------ PV issuer
        if (lane == 0) {
            int J = 0;
            bool ok = true;
            for (int it = 0, t = tile_at(0); t < ntiles && ok; t = tile_at(++it)) {
                const Tile x = tile_of(t);
                for (int j = 0; j < x.nb && ok; j++, J++) {
                    const int pb = J & 1, vs = J % VST;
                    // P(J) is written; p_full(J) also means every warp has
                    // folded PV(J - 2) into its O, so PV buffer pb is free.
                    ok = mbar_wait(bar(bars.p_full[pb]), (J >> 1) & 1, err, 13) &&
                         mbar_wait(bar(bars.v_full[vs]), (J / VST) & 1, err, 14);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t paddr = sP + pb * L::P_BYTES, vaddr = sV + vs * L::V_BYTES;
                    const uint32_t d_pv = tmem + (pb ? TM_PV1 : TM_PV0);
#pragma unroll
                    for (int kk = 0; kk < BLK / 32; kk++)
                        umma_f8(d_pv, smem_desc(paddr + kk * 32, 1024, SWZ_128B),
                                smem_desc(vaddr + kk * 32, 1024, SWZ_128B), IDESC_PV, kk > 0);
                    tc_commit(bar(bars.v_empty[vs]));
                    tc_commit(bar(bars.p_free[pb]));
                }
            }
            tc_commit(bar(bars.pv_done));
            mbar_wait(bar(bars.pv_done), 0, err, 16, false);
        }
    } else {
        // ------------------------------------------------------------ softmax + correction
        const int quarter = warp & 3, sub = warp >> 2;
        const int half = lane >> 4;                             // 0: keys 0-63, 1: keys 64-127
        const int r = quarter * 32 + sub * 16 + (lane & 15);    // query row in the tile = TMEM lane
        const uint32_t lane_base = (uint32_t)(quarter * 32 + sub * 16) << 16;
        const uint32_t prow = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
        int J = 0;  // this CTA's blocks so far
        bool ok = true;
        // This lane's query scale and first key scale of tile t, loaded
        // before the previous tile's epilogue so that their latency is not
        // exposed when the tile's first S (usually computed already) is read.
        auto first_scales = [&](int t, float& q_s, float& k_s) {
            if (t >= ntiles) return;
            const Tile x = tile_of(t);
            const int row_ws = (PARTIAL ? q_tile0 * 128 : 0) + x.qt * 128 + r;
            q_s = __ldg(q_scale + (long long)x.bh_q * (g.tq_pad / QGROUP) + row_ws / QGROUP);
            const int i0 = half < nkb64_seg ? half : 0;
            k_s = __ldg(k_scale + (long long)x.bh_kv * nkb64 + k_key0 / KBLOCK + i0);
        };
        // (measured: faster for dense causal and non-causal segment tiles,
        // slower for dense non-causal (C3: 5.97 vs 5.80 ms) and causal
        // segment tiles, which keep loading them at tile start)
        constexpr bool PREFETCH = CAUSAL != PARTIAL;
        float qs_next = 0.f, ks_next = 0.f;
        if (PREFETCH) first_scales(tile_at(0), qs_next, ks_next);
        for (int it = 0, t = tile_at(0); t < ntiles && ok; t = tile_at(++it)) {
        const Tile tl = tile_of(t);
        const int bh_q = tl.bh_q, bh_kv = tl.bh_kv, qt = tl.qt, nb = tl.nb;
        const int qrow = tl.g0 + r;                             // key position of this row (masking)
        const int qrow_ws = (PARTIAL ? q_tile0 + qt : qt) * 128 + r;  // within the workspace
        const float qs =
            PREFETCH ? qs_next : __ldg(q_scale + (long long)bh_q * (g.tq_pad / QGROUP) + qrow_ws / QGROUP);
        const float* ksc = k_scale + (long long)bh_kv * nkb64 + k_key0 / KBLOCK;
        float o[DH];
#pragma unroll
        for (int c = 0; c < DH; c++) o[c] = 0.f;
        float m = -1.0e30f, l = 0.f, alpha_prev = 0.f;
        auto kscale = [&](int jb) {
            const int i = 2 * jb + half;
            return __ldg(ksc + (i < nkb64_seg ? i : 2 * jb));
        };
        float ks = PREFETCH ? ks_next : kscale(0);
        // O = O * a + PV[block jj] for this lane's D/2 columns: the second
        // level of the FP32 accumulation (each block's PV starts from zero).
        // Waiting for p_free[jj % 2] (committed after PV(jj)) also frees
        // the P buffer of block jj + 2.
        // Barriers tested early (a try_wait issued well before its result is
        // needed, so that its latency stays off the softmax warps' path):
        // pv_ready for the fold's PV, s_ready for the next block's S.
        bool pv_ready = false, s_ready = false;
        auto correct = [&](int jj, float a) -> bool {
            const int pb = jj & 1;
            if (!__all_sync(0xffffffffu, pv_ready) && !warp_wait(bar(bars.p_free[pb]), (jj >> 1) & 1, err, 31))
                return false;
            tc_fence_after();
            const uint64_t a2 = pk2(a, a);
#pragma unroll
            for (int c = 0; c < DH; c += 32) {
                uint32_t pv[32];
                tmem_ld16x2<DH>(tmem + lane_base + (pb ? TM_PV1 : TM_PV0) + c, pv);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    upk2(fma2(pk2(o[c + e], o[c + e + 1]), a2,
                              pk2(__uint_as_float(pv[e]), __uint_as_float(pv[e + 1]))),
                         o[c + e], o[c + e + 1]);
                }
            }
            return true;
        };
        for (int j = 0; j < nb; j++, J++) {
            const int sb = J & 1;
            const float sc = qs * ks;
            if (j + 1 < nb) ks = kscale(j + 1);
            if (!__all_sync(0xffffffffu, s_ready) && !warp_wait(bar(bars.s_full[sb]), (J >> 1) & 1, err, 20)) {
                ok = false;
                break;
            }
            s_ready = false;
            tc_fence_after();
            uint32_t sr[64];
            {
                uint32_t (&c0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[0]);
                uint32_t (&c1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32]);
                const uint32_t ts = tmem + lane_base + (sb ? TM_S1 : TM_S0);
                tmem_ld16x2<64>(ts, c0);
                tmem_ld16x2<64>(ts + 32, c1);
                tmem_wait_ld();
            }
            // x: the float 1.5 * 2^23 + S (dense), or the log2 logit with the
            // merge bias (merged); masked keys -inf.
            float x[64];
            const int key0 = j * BLK + half * 64;
            if (MERGE) {
                // this lane's 64 key biases as 16-byte loads (key0 and
                // tk_pad are multiples of 64, the workspace 256-byte aligned)
                const float c0 = -MAGIC_F * sc;
                const bool in = key0 < g.tk_pad;
                const float4* kb4 = reinterpret_cast<const float4*>(kbias + (in ? key0 : 0));
#pragma unroll
                for (int c = 0; c < 64; c += 4) {
                    const float ninf = __int_as_float(0xff800000);
                    const float4 kb = in ? __ldg(kb4 + c / 4) : make_float4(ninf, ninf, ninf, ninf);
                    x[c] = fmaf(__uint_as_float(sr[c]), sc, kb.x + c0);
                    x[c + 1] = fmaf(__uint_as_float(sr[c + 1]), sc, kb.y + c0);
                    x[c + 2] = fmaf(__uint_as_float(sr[c + 2]), sc, kb.z + c0);
                    x[c + 3] = fmaf(__uint_as_float(sr[c + 3]), sc, kb.w + c0);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; c++) x[c] = __uint_as_float(sr[c]);
            }
            if (j * BLK + BLK > g.tk || (CAUSAL && j * BLK + BLK > tl.g0)) {
#pragma unroll
                for (int c = 0; c < 64; c++) {
                    const int key = key0 + c;
                    if (key >= g.tk || (CAUSAL && key > qrow)) x[c] = __int_as_float(0xff800000);
                }
            }
            float ma = x[0], mb = x[32];
#pragma unroll
            for (int c = 1; c < 31; c += 2) {
                ma = fmax3(ma, x[c], x[c + 1]);
                mb = fmax3(mb, x[32 + c], x[32 + c + 1]);
            }
            float pm = fmax3(ma, mb, fmaxf(x[31], x[63]));
            if (!MERGE) pm = fmaf(pm, sc, -MAGIC_F * sc);  // -inf stays -inf
            const float mnew = fmax3(m, pm, __shfl_xor_sync(0xffffffffu, pm, 16));
            const float alpha = ex2(m - mnew);
            m = mnew;
            // P = 448 * 2^(x - m) as E4M3 into the swizzled P tile (buffer
            // sb is free: PV(j - 2) is done, see correct()).
            const uint32_t prow_addr = sP + sb * L::P_BYTES + prow;
            const float off = MERGE ? LOG2_448 - mnew : LOG2_448 - mnew - MAGIC_F * sc;
            const uint64_t sc2 = pk2(MERGE ? 1.0f : sc, MERGE ? 1.0f : sc), off2 = pk2(off, off);
            uint64_t sum2a = pk2(0.f, 0.f), sum2b = sum2a;
#pragma unroll
            for (int c16 = 0; c16 < 4; c16++) {
                float p[16];
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                    float y0, y1;
                    upk2(fma2(pk2(x[c16 * 16 + e], x[c16 * 16 + e + 1]), sc2, off2), y0, y1);
                    if (e < exp_poly<D>()) {
                        exp2_poly2(y0, y1, p[e], p[e + 1]);
                    } else {
                        p[e] = ex2(y0);
                        p[e + 1] = ex2(y1);
                    }
                    if ((e >> 1) & 1)
                        sum2b = add2(sum2b, pk2(p[e], p[e + 1]));
                    else
                        sum2a = add2(sum2a, pk2(p[e], p[e + 1]));
                }
                uint32_t w[4];
#pragma unroll
                for (int q4 = 0; q4 < 4; q4++) w[q4] = e4m3x4(p[4 * q4], p[4 * q4 + 1], p[4 * q4 + 2], p[4 * q4 + 3]);
                // the fold's PV (block J - 1) is usually done by now
                if (c16 == 1 && j >= 1) pv_ready = mbar_try(bar(bars.p_free[(J - 1) & 1]), ((J - 1) >> 1) & 1);
                const int chunk = half * 4 + c16;
                const uint32_t a = prow_addr + (uint32_t)(((chunk ^ (r & 7)) & 7) << 4);
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                             "r"(w[3])
                             : "memory");
            }
            float s0, s1, s2, s3;
            upk2(sum2a, s0, s1);
            upk2(sum2b, s2, s3);
            l = fmaf(l, alpha, (s0 + s1) + (s2 + s3));
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(bars.p_full[sb]));  // one arrival per warp
            // the next block's S is usually finished during this block
            if (j + 1 < nb) s_ready = mbar_try(bar(bars.s_full[(J + 1) & 1]), ((J + 1) >> 1) & 1);
            // fold the previous block's PV into O while this block's PV runs
            if (j >= 1 && !correct(J - 1, alpha_prev)) {
                ok = false;
                break;
            }
            pv_ready = false;
            alpha_prev = alpha;
        }
        if (ok) ok = correct(J - 1, alpha_prev);  // the tile's last block
        if (PREFETCH) first_scales(tile_at(it + 1), qs_next, ks_next);  // (latency covered by the epilogue)
        if (ok && !PARTIAL && D == 64) {
            // out = O / l * v_scale + v_mean for this lane's D/2 columns,
            // written (bf16) into the warp's staging rows, then stored to
            // the output four whole rows per warp instruction (D = 64: a
            // tile's epilogue is a larger share of its few key blocks; at
            // D = 128 the direct stores below measured faster)
            const float inv = 1.0f / (l + __shfl_xor_sync(0xffffffffu, l, 16));
            const float4* vmean4 = reinterpret_cast<const float4*>(stats + (long long)bh_kv * 4 * D + D + half * DH);
            const float4* vscale4 = vmean4 + D / 4;
            uint8_t* stage = dyn_smem + (sbase - smem_u32(dyn_smem)) + L::STAGE_OFF + (warp * 16) * L::STAGE_ROW;
#pragma unroll
            for (int c = 0; c < DH; c += 8) {
                const float4 s0 = __ldg(vscale4 + c / 4), s1 = __ldg(vscale4 + c / 4 + 1);
                const float4 m0 = __ldg(vmean4 + c / 4), m1 = __ldg(vmean4 + c / 4 + 1);
                const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
                uint32_t w[4];
#pragma unroll
                for (int e2 = 0; e2 < 4; e2++) {
                    const int d = c + 2 * e2;
                    const float y0 = fmaf(o[d] * inv, sv[2 * e2], mv[2 * e2]);
                    const float y1 = fmaf(o[d + 1] * inv, sv[2 * e2 + 1], mv[2 * e2 + 1]);
                    w[e2] = pack_bf16x2(y0, y1);
                }
                *reinterpret_cast<uint4*>(stage + (lane & 15) * L::STAGE_ROW + (half * DH + c) * 2) =
                    make_uint4(w[0], w[1], w[2], w[3]);
            }
            __syncwarp();
            constexpr int CPR = 2 * D / 16, RPI = 32 / CPR;  // 16-byte chunks per row, rows per instruction
            const int row0_ws = qrow_ws - (lane & 15);       // the warp's first row
            uint16_t* obase = out + (long long)(bh_q / g.heads) * g.o_sb + (long long)(bh_q % g.heads) * g.o_sh;
#pragma unroll
            for (int i = 0; i < 16; i += RPI) {
                const int rr = i + lane / CPR, cc = lane % CPR;
                if (row0_ws + rr < g.tokens)
                    *reinterpret_cast<uint4*>(obase + (long long)(row0_ws + rr) * g.o_st + cc * 8) =
                        *reinterpret_cast<const uint4*>(stage + rr * L::STAGE_ROW + cc * 16);
            }
            __syncwarp();  // the staging rows are free for the next tile
        }
        if (ok && !PARTIAL && D == 128) {
            // out = O / l * v_scale + v_mean for this lane's D/2 columns
            const float inv = 1.0f / (l + __shfl_xor_sync(0xffffffffu, l, 16));
            const float* vmean = stats + (long long)bh_kv * 4 * D + D + half * DH;
            const float* vscale = vmean + D;
            uint16_t* orow =
                out + (long long)(bh_q / g.heads) * g.o_sb + (long long)qrow_ws * g.o_st +
                (long long)(bh_q % g.heads) * g.o_sh + half * DH;
            if (qrow_ws < g.tokens) {
#pragma unroll
                for (int c = 0; c < DH; c += 8) {
                    uint32_t w[4];
#pragma unroll
                    for (int e2 = 0; e2 < 4; e2++) {
                        const int d = c + 2 * e2;
                        const float y0 = fmaf(o[d] * inv, __ldg(vscale + d), __ldg(vmean + d));
                        const float y1 = fmaf(o[d + 1] * inv, __ldg(vscale + d + 1), __ldg(vmean + d + 1));
                        w[e2] = pack_bf16x2(y0, y1);
                    }
                    *reinterpret_cast<uint4*>(orow + c) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
        if (ok && PARTIAL) {
            // this segment's y = O / l * v_scale + v_mean and its log2
            // denominator, merged into (acc, lse): acc = (acc w_old + y w_new)
            // / (w_old + w_new) with w = 2^(lse - max), lse = log2 of the sum
            const float lt = l + __shfl_xor_sync(0xffffffffu, l, 16);
            const float inv = 1.0f / lt;
            const float lse_new = m + log2f(lt) - LOG2_448;
            float* lrow = lse + (long long)bh_q * g.tokens + qrow_ws;
            const float lse_old = g.cp_first ? __int_as_float(0xff800000) : *lrow;
            const float mx = fmaxf(lse_old, lse_new);
            const float w_old = lse_old == __int_as_float(0xff800000) ? 0.f : exp2f(lse_old - mx);
            const float w_new = exp2f(lse_new - mx);
            const float s_inv = 1.0f / (w_old + w_new);
            const float a_old = w_old * s_inv, a_new = w_new * inv * s_inv;
            const float* vmean = stats + (long long)bh_kv * 4 * D + D + half * DH;
            const float* vscale = vmean + D;
            float* arow = acc + (long long)(bh_q / g.heads) * g.o_sb + (long long)qrow_ws * g.o_st +
                          (long long)(bh_q % g.heads) * g.o_sh + half * DH;
            if (qrow_ws < g.tokens) {
#pragma unroll
                for (int c = 0; c < DH; c += 4) {
                    float4 x = w_old > 0.f ? *reinterpret_cast<const float4*>(arow + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    x.x = fmaf(x.x, a_old, fmaf(o[c] * a_new, __ldg(vscale + c), __ldg(vmean + c) * w_new * s_inv));
                    x.y = fmaf(x.y, a_old, fmaf(o[c + 1] * a_new, __ldg(vscale + c + 1), __ldg(vmean + c + 1) * w_new * s_inv));
                    x.z = fmaf(x.z, a_old, fmaf(o[c + 2] * a_new, __ldg(vscale + c + 2), __ldg(vmean + c + 2) * w_new * s_inv));
                    x.w = fmaf(x.w, a_old, fmaf(o[c + 3] * a_new, __ldg(vscale + c + 3), __ldg(vmean + c + 3) * w_new * s_inv));
                    *reinterpret_cast<float4*>(arow + c) = x;
                }
            }
            __syncwarp();
            if (half == 0 && qrow_ws < g.tokens) *lrow = mx + log2f(w_old + w_new);
        }
        }  // tiles
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == QK_WARP) tmem_dealloc(tmem, TMEM_COLS);
}

template <int D, bool CAUSAL, bool MERGE, bool PARTIAL, bool GQ = false>
static cudaError_t attend_t(const AttnMaps& maps, const Buffers& buf, const Geom& g, void* out, float* acc, float* lse,
                            int q_tiles, cudaStream_t st) {
    static std::atomic<unsigned> attr_set{0};  // one bit per device ordinal
    auto kern = sp_attn<D, CAUSAL, MERGE, PARTIAL, GQ>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(attr_set.load(std::memory_order_acquire) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem<D>::DYN);
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
    const long long ntiles = (long long)g.batch * g.heads * q_tiles;
    dim3 grid((unsigned)(ntiles < n_sm ? ntiles : n_sm));  // persistent: one CTA per SM
    cudaError_t e = launch_after_previous(kern, grid, dim3(NTHREADS), AttnSmem<D>::DYN, st, maps.q, maps.k, maps.v,
                                          buf.q_scale, buf.k_scale, buf.stats, buf.kbias, (uint16_t*)out, acc, lse,
                                          buf.err, g);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_attend(int d, const AttnMaps& maps, const Buffers& buf, const Geom& g, void* out,
                          cudaStream_t st) {
    const bool merge = g.merge > 1, causal = g.causal != 0;
    const int qt = g.tq_pad / 128;
    if (g.q_split) {  // causal over gathered keys (context parallelism by all-gather)
        if (!causal || merge) return cudaErrorInvalidValue;
        return d == 64 ? attend_t<64, true, false, false, true>(maps, buf, g, out, nullptr, nullptr, qt, st)
                       : attend_t<128, true, false, false, true>(maps, buf, g, out, nullptr, nullptr, qt, st);
    }
    if (d == 64) {
        if (merge) return attend_t<64, false, true, false>(maps, buf, g, out, nullptr, nullptr, qt, st);
        return causal ? attend_t<64, true, false, false>(maps, buf, g, out, nullptr, nullptr, qt, st)
                      : attend_t<64, false, false, false>(maps, buf, g, out, nullptr, nullptr, qt, st);
    }
    if (merge) return attend_t<128, false, true, false>(maps, buf, g, out, nullptr, nullptr, qt, st);
    return causal ? attend_t<128, true, false, false>(maps, buf, g, out, nullptr, nullptr, qt, st)
                  : attend_t<128, false, false, false>(maps, buf, g, out, nullptr, nullptr, qt, st);
}

cudaError_t launch_attend_partial(int d, const AttnMaps& maps, const Buffers& buf, const Geom& g, float* acc,
                                  float* lse, cudaStream_t st) {
    const bool causal = g.causal != 0;
    const int qt = g.q_tiles;  // the segment's query tiles
    if (d == 64)
        return causal ? attend_t<64, true, false, true>(maps, buf, g, nullptr, acc, lse, qt, st)
                      : attend_t<64, false, false, true>(maps, buf, g, nullptr, acc, lse, qt, st);
    return causal ? attend_t<128, true, false, true>(maps, buf, g, nullptr, acc, lse, qt, st)
                  : attend_t<128, false, false, true>(maps, buf, g, nullptr, acc, lse, qt, st);
}

cudaError_t attn_func_attributes(int d, int merge, int* regs, int* local_bytes) {
    cudaFuncAttributes a;
    cudaError_t e = d == 64 ? (merge ? cudaFuncGetAttributes(&a, sp_attn<64, false, true, false>)
                                     : cudaFuncGetAttributes(&a, sp_attn<64, false, false, false>))
                            : (merge ? cudaFuncGetAttributes(&a, sp_attn<128, false, true, false>)
                                     : cudaFuncGetAttributes(&a, sp_attn<128, false, false, false>));
    if (e != cudaSuccess) return e;
    *regs = a.numRegs;
    *local_bytes = (int)a.localSizeBytes;
    return cudaSuccess;
}

int attn_smem_bytes(int d) { return d == 64 ? AttnSmem<64>::DYN : AttnSmem<128>::DYN; }

}  // namespace sp
