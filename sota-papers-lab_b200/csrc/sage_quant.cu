// SageAttention2 quantiser for sm_100a: INT8 Q (one scale per 16 rows, the
// softmax scale and log2(e) folded in), smoothed INT8 K (one scale per 64
// keys), per-channel FP8 E4M3 V, optional KV merging and QK LayerNorm.
//
// The values written are bit-identical to the reference quantiser
// (platform/spl-nn/cuda/sage_quant.cu:59-326): the K/V channel sums follow
// its summation tree (per-thread sequential sums over a 128-token tile,
// an xor butterfly over the lanes that share a channel chunk, a sequential
// sum over the 8 warps, then two interleaved accumulators over the tiles),
// and every rounding happens where it happens there.  What differs is the
// V layout ([b][g][D][tk_pad], keys in order, the K-major operand of the
// tcgen05 PV MMA; sp_export_v rewrites the reference's layout for the bit
// gate) and the separate KV head count (GQA: Q and the K/V statistics run
// as two roles of one launch).
//
// The reference's three launches, all HBM-bound:
//   sp_prep      grid (q_tiles, heads + kv_heads, batch); without its Q
//                role (Q quantised in the QKV GEMM's epilogue) (q_tiles,
//                kv_heads, batch)
//   sp_finalize  grid (kv_heads, batch)
//   sp_quant_kv  grid (tk_pad / 64, kv_heads, batch)
// or, for dense keys without QK LayerNorm (the default), sp_prep_tma: the
// same arithmetic as one persistent TMA-fed launch (see its comment).
#include <mutex>

#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

__device__ __forceinline__ uint4 load8(const uint16_t* p, bool ok) {
    return ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
}

// LayerNorm over one head row whose D channels sit on D/8 consecutive lanes,
// 8 per lane (the reference's sg_layernorm, sage_quant.cu:34-52).  Every lane
// of the warp calls it.  Uses rsqrtf: tolerance-checked, not bit-checked.
template <int D>
__device__ __forceinline__ void layernorm8(float* x, const float* w, const float* bias, int ch, float eps) {
    constexpr int CH = D / 8;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) s += x[e];
#pragma unroll
    for (int o = 1; o < CH; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / D);
    float s2 = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const float t = x[e] - mean;
        s2 += t * t;
    }
#pragma unroll
    for (int o = 1; o < CH; o <<= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float rstd = rsqrtf(s2 * (1.0f / D) + eps);
#pragma unroll
    for (int e = 0; e < 8; e++) x[e] = (x[e] - mean) * rstd * w[ch * 8 + e] + bias[ch * 8 + e];
}

// Q role: one 128-query tile of one q head.
template <int D>
__device__ __forceinline__ void prep_q(const uint16_t* __restrict__ q, const float* __restrict__ ln,
                                       int8_t* __restrict__ q8, float* __restrict__ q_scale, const Geom& g, int tile,
                                       int h, int b) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = QTILE / TPI;
    const int tid = threadIdx.x, lane = tid & 31, ch = tid % CH;
    const long long bh = (long long)b * g.heads + h;
    __shared__ unsigned gmax[QTILE / QGROUP];
    if (tid < QTILE / QGROUP) gmax[tid] = 0u;
    __syncthreads();
    // every load of the tile first; the values are unpacked (and normalised)
    // again for the quantisation pass rather than kept as floats
    uint4 raw[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tok = tile * QTILE + tid / CH + i * TPI;
        raw[i] = load8(q + b * g.q_sb + (long long)tok * g.q_st + h * g.q_sh + ch * 8, tok < g.tokens);
    }
    auto values = [&](int i, float (&f)[8]) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        unpack_bf16x8(raw[i], f);
        if (g.flags & LN_Q) layernorm8<D>(f, ln, ln + D, ch, g.ln_eps);
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (!ok) f[e] = 0.f;
    };
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tl = tid / CH + i * TPI;
        float qv[8];
        values(i, qv);
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(qv[e]));
        // The rows of one warp lie in one 16-row group (32 / CH <= 16 rows).
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) atomicMax(&gmax[tl / QGROUP], __float_as_uint(amax));
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tl = tid / CH + i * TPI;
        const float amax = __uint_as_float(gmax[tl / QGROUP]);
        const float inv = amax > 0.f ? 127.0f / amax : 0.f;
        float f[8];
        values(i, f);
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
        *reinterpret_cast<uint2*>(q8 + (bh * g.tq_pad + tile * QTILE + tl) * D + ch * 8) = w;
    }
    if (tid < QTILE / QGROUP) {
        const float t = __uint_as_float(gmax[tid]) * (1.0f / 127.0f);
        q_scale[bh * (g.tq_pad / QGROUP) + tile * (QTILE / QGROUP) + tid] = t * g.q_mul;
    }
}

// Statistics role: per-channel sum of K, sum / min / max of V over one
// 128-token tile of one kv head, with the reference's reduction tree.
template <int D>
__device__ __forceinline__ void prep_stats(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                           const float* __restrict__ ln, float* __restrict__ part, const Geom& g,
                                           int tile, int h, int b) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = QTILE / TPI;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, ch = tid % CH;
    const long long bh = (long long)b * g.kv_heads + h;
    __shared__ float red[8][4][D];
    float ks[8], vs[8], vmn[8], vmx[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        ks[e] = 0.f;
        vs[e] = 0.f;
        vmn[e] = 3.0e38f;
        vmx[e] = -3.0e38f;
    }
    // K, then V: each a pass of loads issued first, then summed in token
    // order (the K and V statistics are independent accumulations)
    uint4 raw[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tok = tile * QTILE + tid / CH + i * TPI;
        raw[i] = load8(k + b * g.k_sb + (long long)tok * g.k_st + h * g.k_sh + ch * 8, tok < g.tokens);
    }
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        float fk[8];
        unpack_bf16x8(raw[i], fk);
        if (g.flags & LN_K) layernorm8<D>(fk, ln + 2 * D, ln + 3 * D, ch, g.ln_eps);
        if (ok) {
#pragma unroll
            for (int e = 0; e < 8; e++) ks[e] += fk[e];
        }
    }
    // the K sums through the lane butterfly now, so they need no registers
    // during the V pass
#pragma unroll
    for (int o = CH; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; e++) ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], o);
    }
    if (lane < CH) {
#pragma unroll
        for (int e = 0; e < 8; e++) red[warp][0][ch * 8 + e] = ks[e];
    }
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tok = tile * QTILE + tid / CH + i * TPI;
        raw[i] = load8(v + b * g.v_sb + (long long)tok * g.v_st + h * g.v_sh + ch * 8, tok < g.tokens);
    }
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        float fv[8];
        unpack_bf16x8(raw[i], fv);
        if (ok) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                vs[e] += fv[e];
                vmn[e] = fminf(vmn[e], fv[e]);
                vmx[e] = fmaxf(vmx[e], fv[e]);
            }
        }
    }
#pragma unroll
    for (int o = CH; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], o);
            vmn[e] = fminf(vmn[e], __shfl_xor_sync(0xffffffffu, vmn[e], o));
            vmx[e] = fmaxf(vmx[e], __shfl_xor_sync(0xffffffffu, vmx[e], o));
        }
    }
    if (lane < CH) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            red[warp][1][ch * 8 + e] = vs[e];
            red[warp][2][ch * 8 + e] = vmn[e];
            red[warp][3][ch * 8 + e] = vmx[e];
        }
    }
    __syncthreads();
    for (int c = tid; c < 4 * D; c += 256) {
        const int stat = c / D, d = c % D;
        float r = red[0][stat][d];
#pragma unroll
        for (int w = 1; w < 8; w++) {
            const float x = red[w][stat][d];
            r = stat < 2 ? r + x : (stat == 2 ? fminf(r, x) : fmaxf(r, x));
        }
        part[((bh * g.q_tiles + tile) * 4 + stat) * D + d] = r;
    }
}

template <int D>
__global__ void __launch_bounds__(256, 3) sp_prep(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                               const uint16_t* __restrict__ v, const float* __restrict__ ln,
                                               int8_t* __restrict__ q8, float* __restrict__ q_scale,
                                               float* __restrict__ part, const Geom g, int q_role) {
    // grid y: the q heads (Q role, when q_role) and then the kv heads
    const int tile = blockIdx.x, y = blockIdx.y, b = blockIdx.z;
    const int nq = q_role ? g.heads : 0;
    if (y < nq)
        prep_q<D>(q, ln, q8, q_scale, g, tile, y, b);
    else
        prep_stats<D>(k, v, ln, part, g, tile, y - nq, b);
}

// One statistic of one channel over a (batch, kv head)'s tile partials
// (p = the first tile's value, tiles 4 * D floats apart): the tiles summed
// (or min / max-ed) in order as two interleaved accumulators, 16 tiles'
// values loaded before they are combined so that the loads' latency is paid
// once per 16 tiles.  Loads bypass L1: in the one-launch quantiser other CTAs
// of the same launch wrote the partials.
template <int D>
__device__ __forceinline__ float fin_reduce(const float* p, int stat, int q_tiles) {
    float r0 = stat < 2 ? 0.f : (stat == 2 ? 3.0e38f : -3.0e38f);
    float r1 = r0;
    auto acc2 = [&](float x0, float x1) {
        if (stat < 2) {
            r0 += x0;
            r1 += x1;
        } else if (stat == 2) {
            r0 = fminf(r0, x0);
            r1 = fminf(r1, x1);
        } else {
            r0 = fmaxf(r0, x0);
            r1 = fmaxf(r1, x1);
        }
    };
    int t = 0;
    for (; t + 16 <= q_tiles; t += 16) {
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = __ldcg(p + (long long)(t + i) * 4 * D);
#pragma unroll
        for (int i = 0; i < 16; i += 2) acc2(x[i], x[i + 1]);
    }
    for (; t + 1 < q_tiles; t += 2) acc2(__ldcg(p + (long long)t * 4 * D), __ldcg(p + (long long)(t + 1) * 4 * D));
    if (t < q_tiles) {
        const float x0 = __ldcg(p + (long long)t * 4 * D);
        r0 = stat < 2 ? r0 + x0 : (stat == 2 ? fminf(r0, x0) : fmaxf(r0, x0));
    }
    return stat < 2 ? r0 + r1 : (stat == 2 ? fminf(r0, r1) : fmaxf(r0, r1));
}

// Channel d's K mean, V mean, V scale and its reciprocal from its four
// reduced statistics (K sum, V sum, V min, V max).
template <int D>
__device__ __forceinline__ void fin_store(float* o, int d, float ksum, float vsum, float vmin, float vmax,
                                          const Geom& g) {
    const float n = (float)g.tokens;
    const float mk = (g.flags & SMOOTH_K) ? ksum / n : 0.f;
    const float mv = (g.flags & SMOOTH_V) ? vsum / n : 0.f;
    const float amax = fmaxf(vmax - mv, mv - vmin);
    const float scale = amax > 0.f ? amax / g.v_range : 1.0f;
    o[d] = mk;
    o[D + d] = mv;
    o[2 * D + d] = scale;
    o[3 * D + d] = 1.0f / scale;
}

// Per (kv head, batch, 32 channels): K mean, V mean, V scale and its
// reciprocal from the tile partials.  128 threads: (statistic, channel).
template <int D>
__global__ void __launch_bounds__(128) sp_finalize(const float* __restrict__ part, float* __restrict__ stats,
                                                   const Geom g) {
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const long long bh = (long long)b * g.kv_heads + h;
    const int stat = tid >> 5, d = blockIdx.z * 32 + (tid & 31);
    __shared__ float st[4][32];
    st[stat][tid & 31] = fin_reduce<D>(part + bh * g.q_tiles * 4 * D + stat * D + d, stat, g.q_tiles);
    __syncthreads();
    if (tid < 32) fin_store<D>(stats + bh * 4 * D, d, st[0][tid], st[1][tid], st[2][tid], st[3][tid], g);
}

// Members of merged key j within one batch item: the count, the first token
// and the cell's row length (the merge geometry of sage_quant.cu:210-235:
// special tokens and the first dense_frames frames stay single, patch cells
// of merge x merge pool what they cover).
__device__ __forceinline__ int members(const Geom& g, int j, int& base, int& nx) {
    if (g.merge == 1) {
        base = j;
        nx = 1;
        return 1;
    }
    const int dense = g.dense_frames * g.frame_tokens;
    if (j < dense) {
        base = j;
        nx = 1;
        return 1;
    }
    const int f = g.dense_frames + (j - dense) / g.merged_frame, loc = (j - dense) % g.merged_frame;
    if (loc < g.special) {
        base = f * g.frame_tokens + loc;
        nx = 1;
        return 1;
    }
    const int cell = loc - g.special;
    const int gy = cell / g.merged_w, gx = cell % g.merged_w;
    const int y0 = gy * g.merge, x0 = gx * g.merge;
    const int ny = min(g.merge, g.grid_h - y0);
    nx = min(g.merge, g.grid_w - x0);
    base = f * g.frame_tokens + g.special + y0 * g.grid_w + x0;
    return ny * nx;
}

// One 64-key block of one kv head: pool members, subtract the K mean, INT8 K
// with one scale per block; V -> (v - mean) / scale -> E4M3, written
// channel-major ([D][tk_pad]) through a shared-memory transpose.
template <int D>
__device__ __forceinline__ void quant_kv_block(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                               const float* __restrict__ ln, const float* __restrict__ stats,
                                               int8_t* __restrict__ k8, float* __restrict__ k_scale,
                                               uint8_t* __restrict__ v8, float* __restrict__ kbias, const Geom& g,
                                               int blk, int h, int b) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = KBLOCK / TPI;
    const int tid = threadIdx.x, lane = tid & 31, ch = tid % CH;
    const long long bh = (long long)b * g.kv_heads + h;
    const int nblk = g.tk_pad / KBLOCK;
    const int cells = g.merge * g.merge;

    __shared__ unsigned kmax;
    __shared__ __align__(16) uint8_t vt[D][KBLOCK];
    if (tid == 0) kmax = 0u;
    __syncthreads();

    // this thread's channels' K mean, V mean and V 1/scale (read past L1:
    // in the one-launch quantiser another CTA of the launch wrote them)
    float mk[8], mv[8], rv[8];
    {
        const float* st = stats + bh * 4 * D + ch * 8;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            mk[e] = __ldcg(st + e);
            mv[e] = __ldcg(st + D + e);
            rv[e] = __ldcg(st + 3 * D + e);
        }
    }
    if (NI == 4 && g.merge == 1 && !(g.flags & LN_K)) {
        // Dense keys, D = 128: thread (m, ch) takes the 4 consecutive keys
        // 4m .. 4m + 3 of channels ch*8 .. ch*8 + 7, so that each channel's
        // 4 E4M3 bytes form one 32-bit word of the transposed tile (rows of
        // 17 words: at most 4-way bank conflicts).  Every load first; one
        // member per key, so ksum = 0 + k and rc = 1 exactly: the same
        // arithmetic as the general path.
        __shared__ uint32_t vw[D][17];
        const int m = tid / CH;
        uint4 kr[NI], vr[NI];
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const int j = blk * KBLOCK + 4 * m + i;
            const bool ok = j < g.tk;
            kr[i] = load8(k + b * g.k_sb + (long long)j * g.k_st + h * g.k_sh + ch * 8, ok);
            vr[i] = load8(v + b * g.v_sb + (long long)j * g.v_st + h * g.v_sh + ch * 8, ok);
        }
        float kq[NI][8];
        float amx = 0.f;
        uint32_t word[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const bool ok = blk * KBLOCK + 4 * m + i < g.tk;
            float fk[8], fv[8];
            unpack_bf16x8(kr[i], fk);
            unpack_bf16x8(vr[i], fv);
            float vq[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                kq[i][e] = ok ? fmaf(0.f + fk[e], 1.0f, -mk[e]) : 0.f;
                amx = fmaxf(amx, fabsf(kq[i][e]));
                vq[e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const uint32_t two = e4m3x2(vq[e], vq[e + 1]);
                word[e] |= (two & 0xffu) << (8 * i);
                word[e + 1] |= (two >> 8) << (8 * i);
            }
        }
#pragma unroll
        for (int e = 0; e < 8; e++) vw[ch * 8 + e][m] = word[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amx = fmaxf(amx, __shfl_xor_sync(0xffffffffu, amx, o));
        if (lane == 0) atomicMax(&kmax, __float_as_uint(amx));
        __syncthreads();
        const float km = __uint_as_float(kmax);
        const float inv = km > 0.f ? 127.0f / km : 0.f;
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const float* f = kq[i];
            uint2 w;
            w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
            w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
            *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + 4 * m + i) * D + ch * 8) = w;
        }
        if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
        // V: channel d's 64 keys are the 16 words of row d
        for (int c = tid; c < D * 16; c += 256) {
            const int d = c >> 4, w = c & 15;
            *reinterpret_cast<uint32_t*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + 4 * w) = vw[d][w];
        }
        return;
    }
    float kv[NI][8];
    float amax = 0.f;
    if (g.merge == 1 && !(g.flags & LN_K)) {
        // Dense keys: every load of the block first (one member per key, so
        // ksum = 0 + k and rc = 1 exactly: the same arithmetic as below).
        uint4 kr[NI], vr[NI];
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const int j = blk * KBLOCK + tid / CH + i * TPI;
            const bool ok = j < g.tk;
            kr[i] = load8(k + b * g.k_sb + (long long)j * g.k_st + h * g.k_sh + ch * 8, ok);
            vr[i] = load8(v + b * g.v_sb + (long long)j * g.v_st + h * g.v_sh + ch * 8, ok);
        }
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const int kl = tid / CH + i * TPI;
            const bool ok = blk * KBLOCK + kl < g.tk;
            float fk[8], fv[8], vq[8];
            unpack_bf16x8(kr[i], fk);
            unpack_bf16x8(vr[i], fv);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                // 0 + x: the member sum of the general path (it maps -0 to +0)
                kv[i][e] = ok ? fmaf(0.f + fk[e], 1.0f, -mk[e]) : 0.f;
                amax = fmaxf(amax, fabsf(kv[i][e]));
                vq[e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const uint32_t two = e4m3x2(vq[e], vq[e + 1]);
                vt[ch * 8 + e][kl] = (uint8_t)(two & 0xff);
                vt[ch * 8 + e + 1][kl] = (uint8_t)(two >> 8);
            }
        }
    } else
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int kl = tid / CH + i * TPI;
        const int j = blk * KBLOCK + kl;
        const bool ok = j < g.tk;
        int base = 0, nx = 1;
        const int cnt = ok ? members(g, j, base, nx) : 0;
        float ksum[8], vsum[8];
#pragma unroll
        for (int e = 0; e < 8; e++) ksum[e] = vsum[e] = 0.f;
        for (int m = 0; m < cells; m++) {
            const bool mok = m < cnt;
            const int tok = base + (mok ? (m / nx) * g.grid_w + m % nx : 0);
            float fk[8], fv[8];
            unpack_bf16x8(load8(k + b * g.k_sb + (long long)tok * g.k_st + h * g.k_sh + ch * 8, mok), fk);
            unpack_bf16x8(load8(v + b * g.v_sb + (long long)tok * g.v_st + h * g.v_sh + ch * 8, mok), fv);
            if (g.flags & LN_K) layernorm8<D>(fk, ln + 2 * D, ln + 3 * D, ch, g.ln_eps);
            if (mok) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    ksum[e] += fk[e];
                    vsum[e] += fv[e];
                }
            }
        }
        const float rc = cnt > 0 ? 1.0f / (float)cnt : 0.f;
        float vq[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            // fmaf: the contraction nvcc applies to the reference's
            // `ksum * rc - mean` and `(vsum * rc - mv) * inv`.
            kv[i][e] = ok ? fmaf(ksum[e], rc, -mk[e]) : 0.f;
            amax = fmaxf(amax, fabsf(kv[i][e]));
            vq[e] = ok ? fmaf(vsum[e], rc, -mv[e]) * rv[e] : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const uint32_t two = e4m3x2(vq[e], vq[e + 1]);
            vt[ch * 8 + e][kl] = (uint8_t)(two & 0xff);
            vt[ch * 8 + e + 1][kl] = (uint8_t)(two >> 8);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) atomicMax(&kmax, __float_as_uint(amax));
    __syncthreads();

    const float km = __uint_as_float(kmax);
    const float inv = km > 0.f ? 127.0f / km : 0.f;
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int kl = tid / CH + i * TPI;
        const float* f = kv[i];
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
        *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + kl) * D + ch * 8) = w;
    }
    if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
    // V: channel d's 64 keys are 64 contiguous bytes of row d.
    for (int c = tid; c < D * (KBLOCK / 16); c += 256) {
        const int d = c / (KBLOCK / 16), part16 = c % (KBLOCK / 16);
        *reinterpret_cast<uint4*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + part16 * 16) =
            *reinterpret_cast<const uint4*>(&vt[d][part16 * 16]);
    }
    if (g.merge > 1 && b == 0 && h == 0 && tid < KBLOCK) {
        const int j = blk * KBLOCK + tid;
        int base, nx;
        kbias[j] = j < g.tk ? log2f((float)members(g, j, base, nx)) : __int_as_float(0xff800000);
    }
}

template <int D>
__global__ void __launch_bounds__(256) sp_quant_kv(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                                   const float* __restrict__ ln, const float* __restrict__ stats,
                                                   int8_t* __restrict__ k8, float* __restrict__ k_scale,
                                                   uint8_t* __restrict__ v8, float* __restrict__ kbias,
                                                   const Geom g) {
    quant_kv_block<D>(k, v, ln, stats, k8, k_scale, v8, kbias, g, blockIdx.x, blockIdx.y, blockIdx.z);
}

// ---------------------------------------------------------------- one launch
// The three passes above as one persistent launch fed by TMA, for dense keys
// without QK LayerNorm (the other cases keep the three launches).  One CTA
// per SM: a producer warp streams each work item's bf16 input tiles into a
// ring of shared-memory slots (cp.async.bulk.tensor, up to 192 KB in
// flight per SM), eight consumer warps turn them into the outputs with the
// arithmetic of sp_prep / sp_finalize / sp_quant_kv (the same thread-to-
// value mapping, reduction trees and roundings, so the bytes are the same).
// Work items, taken in order from a ticket counter, are laid out in rounds
// r = 0 .. slices + lag - 1 of equal width
//   [ statistics tiles of slice r | a share of the Q tiles | K/V blocks of slice r - lag ]
// (slice = one (batch, kv head); out-of-range items are skipped), so that a
// slice's K and V (2 MB at D = 128, N = 8192) are read again for
// quantisation while its statistics pass has left them in L2.  The CTA that
// finishes a slice's last statistics tile reduces the slice's partials (the
// tree of sp_finalize) and sets the slice's ready flag; a K/V block waits
// for that flag.  No wait can close a cycle: an item only ever waits on
// items with smaller tickets (a K/V block on its slice's statistics tiles,
// which precede it; a ring slot on the items ahead of it in the same ring).
// Every wait is bounded (ERR_TIMEOUT; sites 60-63).
struct PrepSchedule {
    int slices;   // batch * kv_heads
    int ns;       // statistics tiles per slice (q_tiles)
    int nq;       // Q tiles per round
    int nk;       // K/V blocks per slice (tk_pad / 64)
    int lag;      // rounds between a slice's statistics and its K/V blocks
    int q_total;  // Q tiles in all (0: no Q role)
    int width;    // items per round
    int total;    // items in all
};

template <int D>
struct PrepRing {
    static constexpr int TILE = QTILE * D * 2;  // 128 tokens of one head, bf16
    static constexpr int SLOT = 2 * TILE;       // a statistics item: K and V tiles
    static constexpr int NSLOT = 192 * 1024 / SLOT;
    static constexpr int DYN = NSLOT * SLOT + 1024;
    static constexpr int THREADS = 256 + 32;    // eight consumer warps, one producer warp
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// the eight consumer warps only
__device__ __forceinline__ void csync() { named_bar(1, 256); }

__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// prep_q on a tile in shared memory (rows of D bf16; rows past the last
// token were zero-filled by TMA and are zeroed again here, as load8 does).
template <int D>
__device__ __forceinline__ void tile_q(const uint8_t* t, int8_t* __restrict__ q8, float* __restrict__ q_scale,
                                       const Geom& g, int tile, int h, int b, unsigned* gmax) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = QTILE / TPI;
    const int tid = threadIdx.x, lane = tid & 31, ch = tid % CH;
    const long long bh = (long long)b * g.heads + h;
    if (tid < QTILE / QGROUP) gmax[tid] = 0u;
    csync();
    uint4 raw[NI];
#pragma unroll
    for (int i = 0; i < NI; i++) raw[i] = lds16(t + ((tid / CH + i * TPI) * D + ch * 8) * 2);
    auto values = [&](int i, float (&f)[8]) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        unpack_bf16x8(raw[i], f);
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (!ok) f[e] = 0.f;
    };
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tl = tid / CH + i * TPI;
        float qv[8];
        values(i, qv);
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(qv[e]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) atomicMax(&gmax[tl / QGROUP], __float_as_uint(amax));
    }
    csync();
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tl = tid / CH + i * TPI;
        const float amax = __uint_as_float(gmax[tl / QGROUP]);
        const float inv = amax > 0.f ? 127.0f / amax : 0.f;
        float f[8];
        values(i, f);
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
        *reinterpret_cast<uint2*>(q8 + (bh * g.tq_pad + tile * QTILE + tl) * D + ch * 8) = w;
    }
    if (tid < QTILE / QGROUP) {
        const float tq = __uint_as_float(gmax[tid]) * (1.0f / 127.0f);
        q_scale[bh * (g.tq_pad / QGROUP) + tile * (QTILE / QGROUP) + tid] = tq * g.q_mul;
    }
}

// prep_stats on K and V tiles in shared memory; red: [8][4][D] floats.
template <int D>
__device__ __forceinline__ void tile_stats(const uint8_t* kt, const uint8_t* vt, float* __restrict__ part,
                                           const Geom& g, int tile, int h, int b, float* red) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = QTILE / TPI;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, ch = tid % CH;
    const long long bh = (long long)b * g.kv_heads + h;
    float ks[8], vs[8], vmn[8], vmx[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        ks[e] = 0.f;
        vs[e] = 0.f;
        vmn[e] = 3.0e38f;
        vmx[e] = -3.0e38f;
    }
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        float fk[8];
        unpack_bf16x8(lds16(kt + ((tid / CH + i * TPI) * D + ch * 8) * 2), fk);
        if (ok) {
#pragma unroll
            for (int e = 0; e < 8; e++) ks[e] += fk[e];
        }
    }
#pragma unroll
    for (int o = CH; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; e++) ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], o);
    }
    if (lane < CH) {
#pragma unroll
        for (int e = 0; e < 8; e++) red[(warp * 4 + 0) * D + ch * 8 + e] = ks[e];
    }
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
        float fv[8];
        unpack_bf16x8(lds16(vt + ((tid / CH + i * TPI) * D + ch * 8) * 2), fv);
        if (ok) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                vs[e] += fv[e];
                vmn[e] = fminf(vmn[e], fv[e]);
                vmx[e] = fmaxf(vmx[e], fv[e]);
            }
        }
    }
#pragma unroll
    for (int o = CH; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], o);
            vmn[e] = fminf(vmn[e], __shfl_xor_sync(0xffffffffu, vmn[e], o));
            vmx[e] = fmaxf(vmx[e], __shfl_xor_sync(0xffffffffu, vmx[e], o));
        }
    }
    if (lane < CH) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            red[(warp * 4 + 1) * D + ch * 8 + e] = vs[e];
            red[(warp * 4 + 2) * D + ch * 8 + e] = vmn[e];
            red[(warp * 4 + 3) * D + ch * 8 + e] = vmx[e];
        }
    }
    csync();
    for (int c = tid; c < 4 * D; c += 256) {
        const int stat = c / D, d = c % D;
        float r = red[stat * D + d];
#pragma unroll
        for (int w = 1; w < 8; w++) {
            const float x = red[(w * 4 + stat) * D + d];
            r = stat < 2 ? r + x : (stat == 2 ? fminf(r, x) : fmaxf(r, x));
        }
        part[((bh * g.q_tiles + tile) * 4 + stat) * D + d] = r;
    }
}

// quant_kv_block's dense paths (one member per key) on 64-key K and V tiles
// in shared memory; scratch: at least D * 17 words.
template <int D>
__device__ __forceinline__ void tile_quant_kv(const uint8_t* kt, const uint8_t* vt, const float* __restrict__ stats,
                                              int8_t* __restrict__ k8, float* __restrict__ k_scale,
                                              uint8_t* __restrict__ v8, const Geom& g, int blk, int h, int b,
                                              uint32_t* scratch, unsigned* kmax) {
    constexpr int CH = D / 8, TPI = 256 / CH, NI = KBLOCK / TPI;
    const int tid = threadIdx.x, lane = tid & 31, ch = tid % CH;
    const long long bh = (long long)b * g.kv_heads + h;
    const int nblk = g.tk_pad / KBLOCK;
    if (tid == 0) *kmax = 0u;
    float mk[8], mv[8], rv[8];
    {
        const float* st = stats + bh * 4 * D + ch * 8;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            mk[e] = __ldcg(st + e);
            mv[e] = __ldcg(st + D + e);
            rv[e] = __ldcg(st + 3 * D + e);
        }
    }
    csync();
    if (NI == 4) {
        // thread (m, ch): keys 4m .. 4m + 3 of channels ch*8 .. ch*8 + 7, each
        // channel's 4 E4M3 bytes one word of the transposed tile
        uint32_t (*vw)[17] = reinterpret_cast<uint32_t (*)[17]>(scratch);
        const int m = tid / CH;
        float kq[NI][8];
        float amx = 0.f;
        uint32_t word[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const bool ok = blk * KBLOCK + 4 * m + i < g.tk;
            float fk[8], fv[8];
            unpack_bf16x8(lds16(kt + ((4 * m + i) * D + ch * 8) * 2), fk);
            unpack_bf16x8(lds16(vt + ((4 * m + i) * D + ch * 8) * 2), fv);
            float vq[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                kq[i][e] = ok ? fmaf(0.f + fk[e], 1.0f, -mk[e]) : 0.f;
                amx = fmaxf(amx, fabsf(kq[i][e]));
                vq[e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const uint32_t two = e4m3x2(vq[e], vq[e + 1]);
                word[e] |= (two & 0xffu) << (8 * i);
                word[e + 1] |= (two >> 8) << (8 * i);
            }
        }
#pragma unroll
        for (int e = 0; e < 8; e++) vw[ch * 8 + e][m] = word[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amx = fmaxf(amx, __shfl_xor_sync(0xffffffffu, amx, o));
        if (lane == 0) atomicMax(kmax, __float_as_uint(amx));
        csync();
        const float km = __uint_as_float(*kmax);
        const float inv = km > 0.f ? 127.0f / km : 0.f;
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const float* f = kq[i];
            uint2 w;
            w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
            w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
            *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + 4 * m + i) * D + ch * 8) = w;
        }
        if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
        for (int c = tid; c < D * 16; c += 256) {
            const int d = c >> 4, w = c & 15;
            *reinterpret_cast<uint32_t*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + 4 * w) = vw[d][w];
        }
        return;
    }
    uint8_t (*vtr)[KBLOCK] = reinterpret_cast<uint8_t (*)[KBLOCK]>(scratch);
    float kv[NI][8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int kl = tid / CH + i * TPI;
        const bool ok = blk * KBLOCK + kl < g.tk;
        float fk[8], fv[8], vq[8];
        unpack_bf16x8(lds16(kt + (kl * D + ch * 8) * 2), fk);
        unpack_bf16x8(lds16(vt + (kl * D + ch * 8) * 2), fv);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            kv[i][e] = ok ? fmaf(0.f + fk[e], 1.0f, -mk[e]) : 0.f;
            amax = fmaxf(amax, fabsf(kv[i][e]));
            vq[e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const uint32_t two = e4m3x2(vq[e], vq[e + 1]);
            vtr[ch * 8 + e][kl] = (uint8_t)(two & 0xff);
            vtr[ch * 8 + e + 1][kl] = (uint8_t)(two >> 8);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) atomicMax(kmax, __float_as_uint(amax));
    csync();
    const float km = __uint_as_float(*kmax);
    const float inv = km > 0.f ? 127.0f / km : 0.f;
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int kl = tid / CH + i * TPI;
        const float* f = kv[i];
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv);
        *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + kl) * D + ch * 8) = w;
    }
    if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
    for (int c = tid; c < D * (KBLOCK / 16); c += 256) {
        const int d = c / (KBLOCK / 16), part16 = c % (KBLOCK / 16);
        *reinterpret_cast<uint4*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + part16 * 16) =
            *reinterpret_cast<const uint4*>(&vtr[d][part16 * 16]);
    }
}

// Item kinds of the one-launch schedule.
enum : int { ITEM_NONE = 0, ITEM_STATS = 1, ITEM_Q = 2, ITEM_KV = 3 };

__device__ __forceinline__ int item_kind(const PrepSchedule& ps, int item, int& r, int& o) {
    r = item / ps.width;
    o = item % ps.width;
    if (o < ps.ns) return r < ps.slices ? ITEM_STATS : ITEM_NONE;
    if (o < ps.ns + ps.nq) return r * ps.nq + (o - ps.ns) < ps.q_total ? ITEM_Q : ITEM_NONE;
    const int sl = r - ps.lag;
    return sl >= 0 && sl < ps.slices ? ITEM_KV : ITEM_NONE;
}

template <int D>
__global__ void __launch_bounds__(PrepRing<D>::THREADS, 1)
    sp_prep_tma(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Buffers buf, const Geom g, const PrepSchedule ps) {
    using R = PrepRing<D>;
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full[R::NSLOT], empty[R::NSLOT];
    __shared__ int slot_item[R::NSLOT];
    __shared__ __align__(16) float scratch[8 * 4 * D];  // statistics tree or the V transpose
    __shared__ float s_red[4][D];
    __shared__ unsigned s_small[QTILE / QGROUP + 1];
    __shared__ int s_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const uint8_t* ring = dyn_smem + (base - smem_u32(dyn_smem));
    uint32_t* ticket = buf.ctl;
    uint32_t* done = buf.ctl + 1;
    uint32_t* tiles_done = buf.ctl + 2;
    uint32_t* ready = buf.ctl + 2 + ps.slices;
    auto bar = [](uint64_t& x) { return smem_u32(&x); };
    if (tid == 0) {
        for (int i = 0; i < R::NSLOT; i++) {
            mbar_init(bar(full[i]), 1);
            mbar_init(bar(empty[i]), 8);  // one arrival per consumer warp
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 8) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&map_k);
            tma_prefetch_desc(&map_v);
            if (ps.q_total) tma_prefetch_desc(&map_q);
            int n = 0;  // slots filled
            bool ok = true;
            for (;;) {
                int item = (int)atomicAdd(ticket, 1u), r = 0, o = 0;
                int kind = ITEM_NONE;
                if (item < ps.total) {
                    kind = item_kind(ps, item, r, o);
                    if (kind == ITEM_NONE) continue;
                } else {
                    item = -1;  // the end
                }
                const int s = n % R::NSLOT;
                if (n >= R::NSLOT && !(ok = mbar_wait(bar(empty[s]), ((n / R::NSLOT) - 1) & 1, buf.err, 61))) break;
                slot_item[s] = item;
                const uint32_t dst = base + s * R::SLOT, fb = bar(full[s]);
                if (kind == ITEM_STATS) {
                    const int h = r % g.kv_heads, b = r / g.kv_heads, t0 = o * QTILE;
                    mbar_expect_tx(fb, 2 * R::TILE);
                    tma_load_4d(dst, &map_k, fb, 0, h, t0, b);
                    tma_load_4d(dst + R::TILE / 2, &map_k, fb, 0, h, t0 + 64, b);
                    tma_load_4d(dst + R::TILE, &map_v, fb, 0, h, t0, b);
                    tma_load_4d(dst + R::TILE + R::TILE / 2, &map_v, fb, 0, h, t0 + 64, b);
                } else if (kind == ITEM_Q) {
                    const int qi = r * ps.nq + (o - ps.ns);
                    const int tile = qi % g.q_tiles, rest = qi / g.q_tiles;
                    const int h = rest % g.heads, b = rest / g.heads, t0 = tile * QTILE;
                    mbar_expect_tx(fb, R::TILE);
                    tma_load_4d(dst, &map_q, fb, 0, h, t0, b);
                    tma_load_4d(dst + R::TILE / 2, &map_q, fb, 0, h, t0 + 64, b);
                } else if (kind == ITEM_KV) {
                    const int sl = r - ps.lag, blk = o - ps.ns - ps.nq;
                    const int h = sl % g.kv_heads, b = sl / g.kv_heads;
                    mbar_expect_tx(fb, R::TILE);
                    tma_load_4d(dst, &map_k, fb, 0, h, blk * KBLOCK, b);
                    tma_load_4d(dst + R::TILE / 2, &map_v, fb, 0, h, blk * KBLOCK, b);
                } else {
                    mbar_arrive(fb);  // the end marker: no bytes
                }
                n++;
                if (item < 0) break;
            }
            // every load this warp issued has landed before it leaves
            for (int s = 0; s < R::NSLOT && s < n; s++) {
                const int last = s + ((n - 1 - s) / R::NSLOT) * R::NSLOT;
                mbar_wait(bar(full[s]), (last / R::NSLOT) & 1, buf.err, 62, false);
            }
            (void)ok;
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    for (int n = 0;; n++) {
        const int s = n % R::NSLOT;
        if (!warp_all_wait(bar(full[s]), (n / R::NSLOT) & 1, buf.err, 60)) break;
        const int item = slot_item[s];
        if (item < 0) break;
        const uint8_t* slot = ring + s * R::SLOT;
        int r = 0, o = 0;
        const int kind = item_kind(ps, item, r, o);
        csync();  // the previous item's shared scratch is free
        if (kind == ITEM_STATS) {
            const int h = r % g.kv_heads, b = r / g.kv_heads;
            tile_stats<D>(slot, slot + R::TILE, buf.part, g, o, h, b, scratch);
            __threadfence();
            csync();
            if (tid == 0) s_flag = atomicAdd(tiles_done + r, 1u) == (uint32_t)(ps.ns - 1);
            csync();
            if (s_flag) {
                // the slice's last tile: its statistics, as sp_finalize computes them
                __threadfence();
                const long long bh = (long long)b * g.kv_heads + h;
                for (int c = tid; c < 4 * D; c += 256) {
                    const int stat = c / D, d = c % D;
                    s_red[stat][d] = fin_reduce<D>(buf.part + bh * g.q_tiles * 4 * D + stat * D + d, stat, g.q_tiles);
                }
                csync();
                for (int d = tid; d < D; d += 256)
                    fin_store<D>(buf.stats + bh * 4 * D, d, s_red[0][d], s_red[1][d], s_red[2][d], s_red[3][d], g);
                __threadfence();
                csync();
                if (tid == 0) st_release_gpu(ready + r, 1u);
            }
        } else if (kind == ITEM_Q) {
            const int qi = r * ps.nq + (o - ps.ns);
            const int tile = qi % g.q_tiles, rest = qi / g.q_tiles;
            tile_q<D>(slot, buf.q8, buf.q_scale, g, tile, rest % g.heads, rest / g.heads, s_small);
        } else {
            const int sl = r - ps.lag, blk = o - ps.ns - ps.nq;
            if (tid == 0) {
                int ok = 1;
                if (ld_acquire_gpu(ready + sl) == 0u) {
                    const unsigned long long t0 = globaltimer();
                    for (uint32_t i = 1;; ++i) {
                        __nanosleep(128);
                        if (ld_acquire_gpu(ready + sl) != 0u) break;
                        if ((i & 63u) == 0 &&
                            (globaltimer() - t0 > WAIT_LIMIT_NS || i >= WAIT_MAX_TRIES || ld_volatile(buf.err) != 0)) {
                            atomicOr(buf.err, ERR_TIMEOUT | (63u << ERR_SITE_SHIFT));
                            ok = 0;
                            break;
                        }
                    }
                }
                s_flag = ok;
            }
            csync();
            if (s_flag)
                tile_quant_kv<D>(slot, slot + R::TILE / 2, buf.stats, buf.k8, buf.k_scale, buf.v8, g, blk,
                                 sl % g.kv_heads, sl / g.kv_heads, reinterpret_cast<uint32_t*>(scratch),
                                 &s_small[QTILE / QGROUP]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(empty[s]));
    }
    // the last CTA out clears the control words for the next launch
    csync();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            for (int i = 0; i < 2 * ps.slices; i++) tiles_done[i] = 0u;
            *ticket = 0u;
            *done = 0u;
            __threadfence();
        }
    }
}

// The reference's V layout for the bit gate: [b][g][tk_pad/64][D][64], keys
// permuted within each 16 by vpos (sage_common.cu:151-155).
__device__ __forceinline__ int vpos(int k) { return ((k >> 1) & 3) * 4 + ((k >> 3) << 1) + (k & 1); }

template <int D>
__global__ void __launch_bounds__(256) sp_export_v(const uint8_t* __restrict__ v8, uint8_t* __restrict__ out,
                                                   const Geom g) {
    const long long n = (long long)g.batch * g.kv_heads * D * g.tk_pad;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
        const long long key = i % g.tk_pad;
        const long long rest = i / g.tk_pad;  // bh * D + d
        const int d = (int)(rest % D);
        const long long bh = rest / D;
        const int blk = (int)(key / KBLOCK), kl = (int)(key % KBLOCK);
        const long long o = ((bh * (g.tk_pad / KBLOCK) + blk) * D + d) * KBLOCK + (kl & ~15) + vpos(kl & 15);
        out[o] = v8[i];
    }
}

template <int D>
static cudaError_t prepare_d(const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                             const PrepMaps* maps, const Geom& g, cudaStream_t st) {
    const int q_role = q != nullptr;
    if (maps && buf.ctl && g.merge == 1 && !(g.flags & (LN_Q | LN_K))) {
        using R = PrepRing<D>;
        static int sms = 0;
        static std::once_flag once;
        std::call_once(once, [] {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaFuncSetAttribute(sp_prep_tma<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, R::DYN);
        });
        PrepSchedule ps;
        ps.slices = g.batch * g.kv_heads;
        ps.ns = g.q_tiles;
        ps.nk = g.tk_pad / KBLOCK;
        ps.q_total = q_role ? g.batch * g.heads * g.q_tiles : 0;
        // lag: enough rounds that a slice's statistics tiles were all taken
        // well before its first K/V block is (two rings' worth of items per SM)
        const long long need = 2LL * sms * R::NSLOT;
        ps.lag = 1;
        for (;;) {
            const int rounds = ps.slices + ps.lag;
            ps.nq = (ps.q_total + rounds - 1) / rounds;
            ps.width = ps.ns + ps.nq + ps.nk;
            if (ps.lag >= ps.slices || (long long)ps.lag * ps.width + ps.nq >= need) break;
            ps.lag++;
        }
        ps.total = (ps.slices + ps.lag) * ps.width;
        sp_prep_tma<D><<<sms, R::THREADS, R::DYN, st>>>(maps->q, maps->k, maps->v, buf, g, ps);
        return cudaGetLastError();
    }
    sp_prep<D><<<dim3(g.q_tiles, (q_role ? g.heads : 0) + g.kv_heads, g.batch), 256, 0, st>>>(
        (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, ln, buf.q8, buf.q_scale, buf.part, g, q_role);
    sp_finalize<D><<<dim3(g.kv_heads, g.batch, D / 32), 128, 0, st>>>(buf.part, buf.stats, g);
    sp_quant_kv<D><<<dim3(g.tk_pad / KBLOCK, g.kv_heads, g.batch), 256, 0, st>>>(
        (const uint16_t*)k, (const uint16_t*)v, ln, buf.stats, buf.k8, buf.k_scale, buf.v8, buf.kbias, g);
    return cudaGetLastError();
}

cudaError_t launch_prepare(int d, const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                           const PrepMaps* maps, const Geom& g, cudaStream_t st) {
    if (!q) return cudaErrorInvalidValue;
    return d == 64 ? prepare_d<64>(q, k, v, ln, buf, maps, g, st) : prepare_d<128>(q, k, v, ln, buf, maps, g, st);
}

cudaError_t launch_prepare_kv(int d, const void* k, const void* v, const float* ln, const Buffers& buf,
                              const PrepMaps* maps, const Geom& g, cudaStream_t st) {
    return d == 64 ? prepare_d<64>(nullptr, k, v, ln, buf, maps, g, st)
                   : prepare_d<128>(nullptr, k, v, ln, buf, maps, g, st);
}

// ---------------------------------------------------------------- context parallelism
// (No counterpart in the reference, which runs on one GPU.)  Each rank holds
// part of the sequence; the K/V smoothing statistics must be those of the
// whole sequence, so every rank reduces its tiles' partials to raw sums,
// the ranks combine them, and each finalises the same stats from the result.

// raw[b][g][4][D] = {sum K, sum V, -min V, max V} over this rank's tiles.
template <int D>
__global__ void __launch_bounds__(256) sp_cp_partial(const float* __restrict__ part, float* __restrict__ raw,
                                                     const Geom g) {
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const long long bh = (long long)b * g.kv_heads + h;
    for (int c = tid; c < 4 * D; c += 256) {
        const int stat = c / D, d = c % D;
        const float* p = part + bh * g.q_tiles * 4 * D + stat * D + d;
        float r = stat < 2 ? 0.f : (stat == 2 ? 3.0e38f : -3.0e38f);
        for (int t = 0; t < g.q_tiles; t++) {
            const float x = p[(long long)t * 4 * D];
            r = stat < 2 ? r + x : (stat == 2 ? fminf(r, x) : fmaxf(r, x));
        }
        raw[(bh * 4 + stat) * D + d] = stat == 2 ? -r : r;
    }
}

// The workspace stats from the combined raw statistics of `total` tokens
// (the formulas of sp_finalize).
template <int D>
__global__ void __launch_bounds__(256) sp_cp_finalize(const float* __restrict__ raw, float* __restrict__ stats,
                                                      const Geom g, float total) {
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const long long bh = (long long)b * g.kv_heads + h;
    const float* r = raw + bh * 4 * D;
    for (int d = tid; d < D; d += 256) {
        const float mk = (g.flags & SMOOTH_K) ? r[d] / total : 0.f;
        const float mv = (g.flags & SMOOTH_V) ? r[D + d] / total : 0.f;
        const float amax = fmaxf(r[3 * D + d] - mv, mv + r[2 * D + d]);
        const float scale = amax > 0.f ? amax / g.v_range : 1.0f;
        float* o = stats + bh * 4 * D;
        o[d] = mk;
        o[D + d] = mv;
        o[2 * D + d] = scale;
        o[3 * D + d] = 1.0f / scale;
    }
}

// bf16 out [b][t][h][D] (strides g.o_*) from the fp32 accumulator (dense
// [b][t][h][D]).
template <int D>
__global__ void __launch_bounds__(256) sp_cp_finish(const float* __restrict__ acc, uint16_t* __restrict__ out,
                                                    const Geom g) {
    const long long n8 = (long long)g.batch * g.tokens * g.heads * (D / 8);
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n8; i += (long long)gridDim.x * 256) {
        const int c8 = (int)(i % (D / 8));
        const long long row = i / (D / 8);  // (b * tokens + t) * heads + h
        const int h = (int)(row % g.heads);
        const long long bt = row / g.heads;
        const int t = (int)(bt % g.tokens), b = (int)(bt / g.tokens);
        const float4 x0 = *reinterpret_cast<const float4*>(acc + i * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(acc + i * 8 + 4);
        const uint4 w = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                                   pack_bf16x2(x1.z, x1.w));
        *reinterpret_cast<uint4*>(out + b * g.o_sb + (long long)t * g.o_st + (long long)h * g.o_sh + c8 * 8) = w;
    }
}

template <int D>
static cudaError_t cp_prepare_d(const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                                const Geom& g, float* raw, cudaStream_t st) {
    sp_prep<D><<<dim3(g.q_tiles, g.heads + g.kv_heads, g.batch), 256, 0, st>>>(
        (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, ln, buf.q8, buf.q_scale, buf.part, g, 1);
    sp_cp_partial<D><<<dim3(g.kv_heads, g.batch), 256, 0, st>>>(buf.part, raw, g);
    return cudaGetLastError();
}

cudaError_t launch_cp_prepare(int d, const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                              const Geom& g, float* raw, cudaStream_t st) {
    return d == 64 ? cp_prepare_d<64>(q, k, v, ln, buf, g, raw, st) : cp_prepare_d<128>(q, k, v, ln, buf, g, raw, st);
}

template <int D>
static cudaError_t cp_quant_kv_d(const void* k, const void* v, const float* ln, const Buffers& buf, const Geom& g,
                                 const float* raw, float total, cudaStream_t st) {
    sp_cp_finalize<D><<<dim3(g.kv_heads, g.batch), 256, 0, st>>>(raw, buf.stats, g, total);
    sp_quant_kv<D><<<dim3(g.tk_pad / KBLOCK, g.kv_heads, g.batch), 256, 0, st>>>(
        (const uint16_t*)k, (const uint16_t*)v, ln, buf.stats, buf.k8, buf.k_scale, buf.v8, buf.kbias, g);
    return cudaGetLastError();
}

cudaError_t launch_cp_quant_kv(int d, const void* k, const void* v, const float* ln, const Buffers& buf,
                               const Geom& g, const float* raw, float total, cudaStream_t st) {
    return d == 64 ? cp_quant_kv_d<64>(k, v, ln, buf, g, raw, total, st)
                   : cp_quant_kv_d<128>(k, v, ln, buf, g, raw, total, st);
}

// raw [bg][4][D] from the ranks' combined statistics: entries 0-1 (sums)
// from the SUM all-reduce, 2-3 (-min V, max V) from the MAX all-reduce.
__global__ void __launch_bounds__(256) sp_cp_merge_stats(const float* __restrict__ rsum,
                                                         const float* __restrict__ rmax, float* __restrict__ raw,
                                                         int bg, int d) {
    const int n = bg * 4 * d;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        raw[i] = ((i / d) & 3) < 2 ? rsum[i] : rmax[i];
}

cudaError_t launch_cp_merge_stats(const float* rsum, const float* rmax, float* raw, int bg, int d, cudaStream_t st) {
    const int n = bg * 4 * d;
    sp_cp_merge_stats<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, st>>>(rsum, rmax, raw, bg, d);
    return cudaGetLastError();
}

cudaError_t launch_cp_finish(int d, const float* acc, const Geom& g, void* out, cudaStream_t st) {
    const long long n8 = (long long)g.batch * g.tokens * g.heads * (d / 8);
    const long long want = (n8 + 255) / 256;
    const int blocks = (int)(want < 148ll * 16 ? want : 148ll * 16);
    if (d == 64)
        sp_cp_finish<64><<<blocks, 256, 0, st>>>(acc, (uint16_t*)out, g);
    else
        sp_cp_finish<128><<<blocks, 256, 0, st>>>(acc, (uint16_t*)out, g);
    return cudaGetLastError();
}

cudaError_t launch_export_v(int d, const Buffers& buf, const Geom& g, uint8_t* v8_ref, cudaStream_t st) {
    const long long n = (long long)g.batch * g.kv_heads * d * g.tk_pad;
    const long long want = (n + 255) / 256;
    const int blocks = (int)(want < 148ll * 32 ? want : 148ll * 32);
    if (d == 64)
        sp_export_v<64><<<blocks, 256, 0, st>>>(buf.v8, v8_ref, g);
    else
        sp_export_v<128><<<blocks, 256, 0, st>>>(buf.v8, v8_ref, g);
    return cudaGetLastError();
}

}  // namespace sp

// ---------------------------------------------------------------- fixed scratch for spl_sage_quantize_noalloc
//
// Some callers cannot allocate device memory themselves: a library embedded
// in a host application that owns every byte of device memory through its
// own pool (and forbids raw cudaMalloc, which can also synchronise the
// device and fragment that pool), or code that must not take the allocator
// lock on its hot path.  For them the quantiser's only scratch, the per-tile
// channel statistics, lives in this fixed device array instead of a
// workspace.  It is part of the module image, so every GPU that loads the
// library holds it until the process exits.
namespace sp {

constexpr size_t NOALLOC_PART_FLOATS = size_t(1) << 20;  // 4 MiB of per-tile statistics
static __device__ __align__(256) float g_noalloc_part[NOALLOC_PART_FLOATS];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The driver's cuCtxGetCurrent, looked up once through the runtime (the
// library does not link libcuda).
static CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (CtxGetCurrentFn)p;
    });
    return fn;
}

// Device address of g_noalloc_part on the current device.  In host code the
// array's name is only a host-side stand-in, so its device address is asked
// for once per device (with that device current) and cached together with
// the context it was asked in: a device reset that re-creates the context
// (and reloads the module) makes the next call ask again.
cudaError_t noalloc_part_buffer(float** out) {
    static std::mutex mu;
    static float* addr[64] = {nullptr};
    static CUcontext ctx_of[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    CtxGetCurrentFn get = ctx_get_current_fn();
    CUcontext ctx = nullptr;
    if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    // (a thread with no context bound yet reads NULL: look the address up,
    // which binds the device's primary context, and then read it again)
    if (!addr[dev] || !ctx || ctx != ctx_of[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_part);
        if (e != cudaSuccess) return e;
        if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
        addr[dev] = (float*)p;
        ctx_of[dev] = ctx;
    }
    *out = addr[dev];
    return cudaSuccess;
}

size_t noalloc_part_capacity() { return NOALLOC_PART_FLOATS; }

}  // namespace sp
