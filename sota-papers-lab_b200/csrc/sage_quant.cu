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
// Launches, all HBM-bound:
//   sp_prep             grid (q_tiles, batch * (heads + kv_heads)): every
//                       Q role (none when the QKV GEMM's epilogue quantised
//                       Q), then every K/V statistics role; with a workspace
//                       the CTA that finishes a (batch, kv head)'s last tile
//                       also reduces its statistics
//   sp_finalize         grid (kv_heads, batch, D / 32): that reduction where
//                       there is no workspace counter (the no-allocation call)
//   sp_quant_kv_stream  dense keys without QK LayerNorm: persistent, one
//                       64-key block after another, newest statistics first
//   sp_quant_kv         grid (tk_pad / 64, kv_heads, batch): merged keys, QK
//                       LayerNorm, context parallelism
#include <mutex>

#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

// The transposed V tile at D = 128 (vw[D][17]: per channel, 16 words of four
// keys' E4M3 bytes): key group w of channel d is kept in column
// (w + 2 * (d / 32)) mod 16, so that the 32 lanes of a warp (16 channel
// chunks x 2 key groups) store to 32 different banks (unswizzled, channel
// chunks ch, ch + 4, ch + 8, ch + 12 met in one bank).
__device__ __forceinline__ int vw_col(int w, int d) { return (w + 2 * (d >> 5)) & 15; }

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

// One statistic of one channel over a (batch, kv head)'s tile partials
// (p = the first tile's value, tiles 4 * D floats apart): the tiles summed
// (or min / max-ed) in order as two interleaved accumulators, 16 tiles'
// values loaded before they are combined so that the loads' latency is paid
// once per 16 tiles.  Loads bypass L1: when sp_prep reduces them, other CTAs of
// the same launch wrote the partials.
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

// Q role without QK LayerNorm: one 128-query tile of one q head, warp w
// taking the 16-row scale group w, so that the group's maximum is a warp
// reduction (no shared memory, atomics or block barrier).  Lane l holds
// channels (l % CH) * 8 .. + 7 (CH = D / 8 chunks per row) of rows
// 16 w + (32 / CH) i + l / CH: each load and store instruction of the warp
// covers 32 / CH whole rows.  The group maximum of |x| is taken on the bf16
// values (exact, NaN-ignoring like fmaxf): the same values and roundings as
// prep_q below, in fewer instructions.
template <int D>
__device__ __forceinline__ void prep_q16(const uint16_t* __restrict__ q, int8_t* __restrict__ q8,
                                         float* __restrict__ q_scale, const Geom& g, int tile, int h, int b) {
    constexpr int CH = D / 8, RPI = 32 / CH, NV = QGROUP / RPI;  // rows per instruction, rows per lane
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, ch = lane % CH;
    const int r0 = warp * QGROUP + lane / CH;  // the lane's first row in the tile
    const long long bh = (long long)b * g.heads + h;
    const uint16_t* src = q + b * g.q_sb + h * g.q_sh + ch * 8;
    uint4 raw[NV];
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const int tok = tile * QTILE + r0 + j * RPI;
        raw[j] = load8(src + (long long)tok * g.q_st, tok < g.tokens);
    }
    uint32_t m2 = 0u;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        m2 = bmax2(m2, raw[j].x & 0x7fff7fffu);
        m2 = bmax2(m2, raw[j].y & 0x7fff7fffu);
        m2 = bmax2(m2, raw[j].z & 0x7fff7fffu);
        m2 = bmax2(m2, raw[j].w & 0x7fff7fffu);
    }
    float amax = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    const bool fast = s8_fast(amax);
    int8_t* dst = q8 + (bh * g.tq_pad + tile * QTILE + r0) * D + ch * 8;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        float f[8];
        unpack_bf16x8(raw[j], f);
        // __fmul_rn: the product keeps its own rounding (never fused with
        // s8x4's rounding add; an FMA would break ties such as 63.5)
        uint2 w;
        w.x = s8x4(__fmul_rn(f[0], inv), __fmul_rn(f[1], inv), __fmul_rn(f[2], inv), __fmul_rn(f[3], inv), fast);
        w.y = s8x4(__fmul_rn(f[4], inv), __fmul_rn(f[5], inv), __fmul_rn(f[6], inv), __fmul_rn(f[7], inv), fast);
        *reinterpret_cast<uint2*>(dst + (long long)j * RPI * D) = w;
    }
    if (lane == 0)
        q_scale[bh * (g.tq_pad / QGROUP) + tile * (QTILE / QGROUP) + warp] = (amax * (1.0f / 127.0f)) * g.q_mul;
}

// Q role: one 128-query tile of one q head (any options; QK LayerNorm
// needs a row's channels on consecutive lanes).
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
        const bool fast = s8_fast(amax);
        float f[8];
        values(i, f);
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv, fast);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv, fast);
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
                                           const float* __restrict__ ln, float* __restrict__ part,
                                           float* __restrict__ stats, uint32_t* __restrict__ tiles_done,
                                           const Geom& g, int tile, int h, int b) {
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
    // the K loads and the first NV0 V loads issued together (the rest of V
    // once K's registers are free: all of it would spill at D = 128), then
    // K and V each summed in token order (independent accumulations)
    constexpr int NV0 = NI <= 4 ? NI : NI / 2;
    uint4 raw[NI], rawv[NI];
    auto load_v = [&](int i) {
        const int tok = tile * QTILE + tid / CH + i * TPI;
        rawv[i] = load8(v + b * g.v_sb + (long long)tok * g.v_st + h * g.v_sh + ch * 8, tok < g.tokens);
    };
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int tok = tile * QTILE + tid / CH + i * TPI;
        raw[i] = load8(k + b * g.k_sb + (long long)tok * g.k_st + h * g.k_sh + ch * 8, tok < g.tokens);
    }
#pragma unroll
    for (int i = 0; i < NV0; i++) load_v(i);
    if (g.flags & LN_K) {
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const bool ok = tile * QTILE + tid / CH + i * TPI < g.tokens;
            float fk[8];
            unpack_bf16x8(raw[i], fk);
            layernorm8<D>(fk, ln + 2 * D, ln + 3 * D, ch, g.ln_eps);
            if (ok) {
#pragma unroll
                for (int e = 0; e < 8; e++) ks[e] += fk[e];
            }
        }
    } else {
        // the same sums, in the same order, as packed pairs
        uint64_t k2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < NI; i++) {
            if (tile * QTILE + tid / CH + i * TPI < g.tokens) {
                k2[0] = add2(k2[0], bf2_to_f2(raw[i].x));
                k2[1] = add2(k2[1], bf2_to_f2(raw[i].y));
                k2[2] = add2(k2[2], bf2_to_f2(raw[i].z));
                k2[3] = add2(k2[3], bf2_to_f2(raw[i].w));
            }
        }
#pragma unroll
        for (int p2 = 0; p2 < 4; p2++) upk2(k2[p2], ks[2 * p2], ks[2 * p2 + 1]);
    }
#pragma unroll
    for (int i = NV0; i < NI; i++) load_v(i);
    // the K sums through the lane butterfly now, so they need no registers
    // during the V sums
#pragma unroll
    for (int o = CH; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; e++) ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], o);
    }
    if (lane < CH) {
#pragma unroll
        for (int e = 0; e < 8; e++) red[warp][0][ch * 8 + e] = ks[e];
    }
    {
        // sums as packed pairs (the same order and roundings); minimum and
        // maximum on the bf16 values (exact), starting from +-infinity and
        // clamped to the +-3e38 starting values afterwards
        uint64_t v2[4] = {0ull, 0ull, 0ull, 0ull};
        uint32_t mn[4] = {0x7f807f80u, 0x7f807f80u, 0x7f807f80u, 0x7f807f80u};
        uint32_t mx[4] = {0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u};
#pragma unroll
        for (int i = 0; i < NI; i++) {
            if (tile * QTILE + tid / CH + i * TPI < g.tokens) {
                const uint32_t w[4] = {rawv[i].x, rawv[i].y, rawv[i].z, rawv[i].w};
#pragma unroll
                for (int p2 = 0; p2 < 4; p2++) {
                    v2[p2] = add2(v2[p2], bf2_to_f2(w[p2]));
                    mn[p2] = bmin2(mn[p2], w[p2]);
                    mx[p2] = bmax2(mx[p2], w[p2]);
                }
            }
        }
#pragma unroll
        for (int p2 = 0; p2 < 4; p2++) {
            upk2(v2[p2], vs[2 * p2], vs[2 * p2 + 1]);
            vmn[2 * p2] = fminf(vmn[2 * p2], __uint_as_float(mn[p2] << 16));
            vmn[2 * p2 + 1] = fminf(vmn[2 * p2 + 1], __uint_as_float(mn[p2] & 0xffff0000u));
            vmx[2 * p2] = fmaxf(vmx[2 * p2], __uint_as_float(mx[p2] << 16));
            vmx[2 * p2 + 1] = fmaxf(vmx[2 * p2 + 1], __uint_as_float(mx[p2] & 0xffff0000u));
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
    if (!tiles_done) return;
    // The CTA that finishes the slice's last tile reduces the slice's
    // partials (the tree of sp_finalize) and clears its count for the next
    // launch; sp_finalize then does not run.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(tiles_done + bh, 1u) == (uint32_t)(g.q_tiles - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    float* fr = &red[0][0][0];  // the four reduced statistics, [4][D]
    for (int c = tid; c < 4 * D; c += 256)
        fr[c] = fin_reduce<D>(part + bh * g.q_tiles * 4 * D + (c / D) * D + c % D, c / D, g.q_tiles);
    __syncthreads();
    for (int d = tid; d < D; d += 256) fin_store<D>(stats + bh * 4 * D, d, fr[d], fr[D + d], fr[2 * D + d], fr[3 * D + d], g);
    if (tid == 0) tiles_done[bh] = 0u;
}

// four CTAs per SM at D = 64 (64 registers suffice there), three at D = 128
template <int D>
__global__ void __launch_bounds__(256, D == 64 ? 4 : 3) sp_prep(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                               const uint16_t* __restrict__ v, const float* __restrict__ ln,
                                               int8_t* __restrict__ q8, float* __restrict__ q_scale,
                                               float* __restrict__ part, float* __restrict__ stats,
                                               uint32_t* __restrict__ tiles_done, const Geom g, int q_role) {
    // grid y: the Q role of every (batch, q head) (when q_role), then the
    // statistics role of every (batch, kv head), so that the K and V tiles
    // are the last inputs read (sp_quant_kv reads them again, newest first,
    // while they are still in L2)
    // the next launch (sp_quant_kv_stream) may start once every CTA of this
    // grid has started; it waits for this grid's end before it reads the
    // statistics
    griddep_launch_dependents();
    // this grid may itself start while the kernel before it (the QKV GEMM, the
    // previous attention) finishes: nothing is read or written before its end
    griddep_wait();
    const int tile = blockIdx.x, y = blockIdx.y + blockIdx.z * gridDim.y;
    const int nq = q_role ? g.batch * g.heads : 0;
    if (y >= nq + g.batch * g.kv_heads) return;  // past the roles (grid y split over z)
    if (y < nq)
        if (g.flags & LN_Q)
            prep_q<D>(q, ln, q8, q_scale, g, tile, y % g.heads, y / g.heads);
        else
            prep_q16<D>(q, q8, q_scale, g, tile, y % g.heads, y / g.heads);
    else
        prep_stats<D>(k, v, ln, part, stats, tiles_done, g, tile, (y - nq) % g.kv_heads, (y - nq) / g.kv_heads);
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
        // 17 words, key groups in swizzled columns: vw_col).  Every load first; one
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
        for (int e = 0; e < 8; e++) vw[ch * 8 + e][vw_col(m, ch * 8)] = word[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amx = fmaxf(amx, __shfl_xor_sync(0xffffffffu, amx, o));
        if (lane == 0) atomicMax(&kmax, __float_as_uint(amx));
        __syncthreads();
        const float km = __uint_as_float(kmax);
        const float inv = km > 0.f ? 127.0f / km : 0.f;
        const bool fast = s8_fast(km);
#pragma unroll
        for (int i = 0; i < NI; i++) {
            const float* f = kq[i];
            uint2 w;
            w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv, fast);
            w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv, fast);
            *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + 4 * m + i) * D + ch * 8) = w;
        }
        if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
        // V: channel d's 64 keys are the 16 words of row d, stored 16 keys
        // (four words) at a time
        for (int c = tid; c < D * 4; c += 256) {
            const int d = c >> 2, w = 4 * (c & 3);
            *reinterpret_cast<uint4*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + 4 * w) =
                make_uint4(vw[d][vw_col(w, d)], vw[d][vw_col(w + 1, d)], vw[d][vw_col(w + 2, d)],
                           vw[d][vw_col(w + 3, d)]);
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
    const bool fast = s8_fast(km);
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int kl = tid / CH + i * TPI;
        const float* f = kv[i];
        uint2 w;
        w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv, fast);
        w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv, fast);
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

// Resident sp_quant_kv CTAs per SM the register allocation must allow: the
// kernel waits on its loads (one 64-key K and V block per CTA), so more CTAs
// keep more bytes in flight.
#ifndef SP_QUANT_KV_CTAS
#define SP_QUANT_KV_CTAS 3
#endif
template <int D>
__global__ void __launch_bounds__(256, SP_QUANT_KV_CTAS) sp_quant_kv(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                                   const float* __restrict__ ln, const float* __restrict__ stats,
                                                   int8_t* __restrict__ k8, float* __restrict__ k_scale,
                                                   uint8_t* __restrict__ v8, float* __restrict__ kbias,
                                                   const Geom g) {
    // newest statistics tiles first (reverse of sp_prep's order): their K
    // and V are the likeliest to be in L2 still
    quant_kv_block<D>(k, v, ln, stats, k8, k_scale, v8, kbias, g, gridDim.x - 1 - blockIdx.x,
                      gridDim.y - 1 - blockIdx.y, gridDim.z - 1 - blockIdx.z);
}

// ---------------------------------------------------------------- streaming K/V quantisation
// sp_quant_kv for dense keys without QK LayerNorm (the common case) as a
// persistent kernel: each CTA takes every gridDim.x-th 64-key block (newest
// statistics tiles first, as sp_quant_kv) and copies the next block's K and
// V rows into shared memory with cp.async while it quantises the current
// one, so that loads stay in flight across blocks.  The arithmetic is
// quant_kv_block's dense paths (one member per key), value for value.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D>
struct KvStream {
    static constexpr int ROW = D * 2;                // bytes of one key row of one head
    static constexpr int TILE = KBLOCK * ROW;        // one tensor's 64 keys
    static constexpr int STAGE = 2 * TILE;           // K and V
    static constexpr int DYN = 2 * STAGE + D * 17 * 4 + 16;  // two stages, the V transpose, kmax
};

template <int D>
__global__ void __launch_bounds__(256, D == 64 ? 4 : 3) sp_quant_kv_stream(const uint16_t* __restrict__ k,
                                                             const uint16_t* __restrict__ v,
                                                             const float* __restrict__ stats, int8_t* __restrict__ k8,
                                                             float* __restrict__ k_scale, uint8_t* __restrict__ v8,
                                                             const Geom g) {
    using S = KvStream<D>;
    constexpr int CH = D / 8, TPI = 256 / CH, NI = KBLOCK / TPI;
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    uint32_t* scratch = reinterpret_cast<uint32_t*>(dyn_smem + 2 * S::STAGE);
    unsigned* kmax = reinterpret_cast<unsigned*>(dyn_smem + 2 * S::STAGE + D * 17 * 4);
    const int tid = threadIdx.x, lane = tid & 31, ch = tid % CH;
    const int nblk = g.tk_pad / KBLOCK, total = g.batch * g.kv_heads * nblk;
    auto decode = [&](int item, int& blk, int& h, int& b) {
        const int idx = total - 1 - item;  // newest first
        blk = idx % nblk;
        h = (idx / nblk) % g.kv_heads;
        b = idx / nblk / g.kv_heads;
    };
    auto issue = [&](int item, int stage) {
        int blk, h, b;
        decode(item, blk, h, b);
        const uint32_t base = smem_u32(dyn_smem) + stage * S::STAGE;
        for (int c = tid; c < KBLOCK * CH; c += 256) {
            const int key = c / CH, cc = c % CH, j = blk * KBLOCK + key;
            if (j < g.tk) {  // rows past the end are masked in the arithmetic
                cp_async16(base + key * S::ROW + cc * 16, k + b * g.k_sb + (long long)j * g.k_st + h * g.k_sh + cc * 8);
                cp_async16(base + S::TILE + key * S::ROW + cc * 16,
                           v + b * g.v_sb + (long long)j * g.v_st + h * g.v_sh + cc * 8);
            }
        }
        cp_async_commit();
    };
    int item = blockIdx.x;
    if (item < total) issue(item, 0);  // K and V are inputs of the whole quantiser
    griddep_wait();                    // the statistics come from sp_prep (or sp_finalize)
    for (int n = 0; item < total; item += gridDim.x, n++) {
        if (item + (int)gridDim.x >= total) griddep_launch_dependents();  // this CTA's last block
        int blk, h, b;
        decode(item, blk, h, b);
        const long long bh = (long long)b * g.kv_heads + h;
        // the slice's statistics requested before the wait for its rows, so
        // that the two latencies overlap
        const float4* st = reinterpret_cast<const float4*>(stats + bh * 4 * D + ch * 8);
        const float4 a0 = __ldg(st), a1 = __ldg(st + 1), b0 = __ldg(st + D / 4), b1 = __ldg(st + D / 4 + 1);
        const float4 c0 = __ldg(st + 3 * D / 4), c1 = __ldg(st + 3 * D / 4 + 1);
        if (item + (int)gridDim.x < total) {
            issue(item + gridDim.x, (n + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        if (tid == 0) *kmax = 0u;
        __syncthreads();  // this stage's rows (all threads' copies) have landed
        const uint8_t* kt = dyn_smem + (n & 1) * S::STAGE;
        const uint8_t* vt = kt + S::TILE;
        float mk[8], mv[8], rv[8];
        {
            mk[0] = a0.x; mk[1] = a0.y; mk[2] = a0.z; mk[3] = a0.w; mk[4] = a1.x; mk[5] = a1.y; mk[6] = a1.z; mk[7] = a1.w;
            mv[0] = b0.x; mv[1] = b0.y; mv[2] = b0.z; mv[3] = b0.w; mv[4] = b1.x; mv[5] = b1.y; mv[6] = b1.z; mv[7] = b1.w;
            rv[0] = c0.x; rv[1] = c0.y; rv[2] = c0.z; rv[3] = c0.w; rv[4] = c1.x; rv[5] = c1.y; rv[6] = c1.z; rv[7] = c1.w;
        }
        if constexpr (NI == 4) {
            // thread (m, ch): keys 4m .. 4m + 3 of channels ch*8 .. ch*8 + 7,
            // each channel's 4 E4M3 bytes one word of the transposed tile
            uint32_t (*vw)[17] = reinterpret_cast<uint32_t (*)[17]>(scratch);
            const int m = tid / CH;
            float kq[NI][8];
            float amx = 0.f;
            uint32_t two[NI][4];  // E4M3 pairs (channels 2p, 2p + 1) of each key
            // key i of this thread's four; ok false: a key past the end (zeros)
            auto key = [&](int i, bool ok) {
                float fk[8], fv[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(kt + (4 * m + i) * S::ROW + ch * 16), fk);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(vt + (4 * m + i) * S::ROW + ch * 16), fv);
                float vq[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    // fk - mk is the reference's fma(k, 1, -mean); it differs from
                    // quant_kv_block's (0 + fk) only in the sign of a zero,
                    // which no K byte or maximum sees
                    kq[i][e] = ok ? fk[e] - mk[e] : 0.f;
                    amx = fmaxf(amx, fabsf(kq[i][e]));
                    vq[e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
                }
#pragma unroll
                for (int p2 = 0; p2 < 4; p2++) two[i][p2] = e4m3x2(vq[2 * p2], vq[2 * p2 + 1]);
            };
            if (blk * KBLOCK + KBLOCK <= g.tk) {
#pragma unroll
                for (int i = 0; i < NI; i++) key(i, true);  // a whole block: no key masked
            } else {
#pragma unroll
                for (int i = 0; i < NI; i++) key(i, blk * KBLOCK + 4 * m + i < g.tk);
            }
            // each channel's 4 bytes (keys 4m .. 4m + 3) into one word
            uint32_t word[8];
#pragma unroll
            for (int p2 = 0; p2 < 4; p2++) {
                word[2 * p2] = __byte_perm(__byte_perm(two[0][p2], two[1][p2], 0x0040),
                                           __byte_perm(two[2][p2], two[3][p2], 0x0040), 0x5410);
                word[2 * p2 + 1] = __byte_perm(__byte_perm(two[0][p2], two[1][p2], 0x0051),
                                               __byte_perm(two[2][p2], two[3][p2], 0x0051), 0x5410);
            }
#pragma unroll
            for (int e = 0; e < 8; e++) vw[ch * 8 + e][vw_col(m, ch * 8)] = word[e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amx = fmaxf(amx, __shfl_xor_sync(0xffffffffu, amx, o));
            if (lane == 0) atomicMax(kmax, __float_as_uint(amx));
            __syncthreads();
            const float km = __uint_as_float(*kmax);
            const float inv = km > 0.f ? 127.0f / km : 0.f;
            const bool fast = s8_fast(km);
#pragma unroll
            for (int i = 0; i < NI; i++) {
                const float* f = kq[i];
                uint2 w;
                w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv, fast);
                w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv, fast);
                *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + 4 * m + i) * D + ch * 8) = w;
            }
            if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
            for (int c = tid; c < D * 4; c += 256) {
                const int d = c >> 2, w = 4 * (c & 3);
                *reinterpret_cast<uint4*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + 4 * w) =
                    make_uint4(vw[d][vw_col(w, d)], vw[d][vw_col(w + 1, d)], vw[d][vw_col(w + 2, d)],
                           vw[d][vw_col(w + 3, d)]);
            }
        } else {
            static_assert(NI == 2, "D = 64: two keys per thread");
            // thread (m, ch): keys 2m and 2m + 1 of channels ch*8 .. ch*8 + 7;
            // each channel's two E4M3 bytes one 16-bit element of the
            // transposed tile, whose rows of 33 elements (66 bytes) put the
            // eight channel chunks of a warp's store in different banks
            constexpr int TROW = KBLOCK / 2 + 1;
            uint16_t (*vt16)[TROW] = reinterpret_cast<uint16_t (*)[TROW]>(scratch);
            const int m = tid / CH;
            float kv[NI][8];
            float amax = 0.f;
            float vq[NI][8];
#pragma unroll
            for (int i = 0; i < NI; i++) {
                const int kl = 2 * m + i;
                const bool ok = blk * KBLOCK + kl < g.tk;
                float fk[8], fv[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(kt + kl * S::ROW + ch * 16), fk);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(vt + kl * S::ROW + ch * 16), fv);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    kv[i][e] = ok ? fmaf(0.f + fk[e], 1.0f, -mk[e]) : 0.f;
                    amax = fmaxf(amax, fabsf(kv[i][e]));
                    vq[i][e] = ok ? fmaf(0.f + fv[e], 1.0f, -mv[e]) * rv[e] : 0.f;
                }
            }
#pragma unroll
            for (int e = 0; e < 8; e++) vt16[ch * 8 + e][m] = (uint16_t)e4m3x2(vq[0][e], vq[1][e]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if (lane == 0) atomicMax(kmax, __float_as_uint(amax));
            __syncthreads();
            const float km = __uint_as_float(*kmax);
            const float inv = km > 0.f ? 127.0f / km : 0.f;
            const bool fast = s8_fast(km);
#pragma unroll
            for (int i = 0; i < NI; i++) {
                const int kl = 2 * m + i;
                const float* f = kv[i];
                uint2 w;
                w.x = s8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv, fast);
                w.y = s8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv, fast);
                *reinterpret_cast<uint2*>(k8 + (bh * g.tk_pad + blk * KBLOCK + kl) * D + ch * 8) = w;
            }
            if (tid == 0) k_scale[bh * nblk + blk] = km * (1.0f / 127.0f);
            for (int c = tid; c < D * (KBLOCK / 16); c += 256) {
                const int d = c / (KBLOCK / 16), part16 = c % (KBLOCK / 16);
                const uint16_t* src = &vt16[d][part16 * 8];
                uint4 w;
                w.x = (uint32_t)src[0] | ((uint32_t)src[1] << 16);
                w.y = (uint32_t)src[2] | ((uint32_t)src[3] << 16);
                w.z = (uint32_t)src[4] | ((uint32_t)src[5] << 16);
                w.w = (uint32_t)src[6] | ((uint32_t)src[7] << 16);
                *reinterpret_cast<uint4*>(v8 + (bh * D + d) * (long long)g.tk_pad + blk * KBLOCK + part16 * 16) = w;
            }
        }
        __syncthreads();  // this stage and the transpose are free for the next blocks
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

// sp_prep's grid: x the 128-token tiles, y (split over z past 65535) the
// roles of every batch item.
static dim3 prep_grid(const Geom& g, int q_role) {
    const int roles = g.batch * ((q_role ? g.heads : 0) + g.kv_heads);
    const int y = roles < 65535 ? roles : 65535;
    return dim3(g.q_tiles, y, (roles + y - 1) / y);
}

template <int D>
static cudaError_t prepare_d(const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                             const Geom& g, cudaStream_t st) {
    const int q_role = q != nullptr;
    cudaError_t e0 = launch_after_previous(sp_prep<D>, prep_grid(g, q_role), dim3(256), 0, st, (const uint16_t*)q,
                                           (const uint16_t*)k, (const uint16_t*)v, ln, buf.q8, buf.q_scale, buf.part,
                                           buf.stats, buf.tiles_done, g, q_role);
    if (e0 != cudaSuccess) return e0;
    if (!buf.tiles_done) sp_finalize<D><<<dim3(g.kv_heads, g.batch, D / 32), 128, 0, st>>>(buf.part, buf.stats, g);
    if (g.merge == 1 && !(g.flags & LN_K)) {
        using S = KvStream<D>;
        static int ctas = 0;
        static std::once_flag once;
        std::call_once(once, [] {
            int dev = 0, sms = 0, per = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaFuncSetAttribute(sp_quant_kv_stream<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::DYN);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, sp_quant_kv_stream<D>, 256, S::DYN);
            ctas = sms * (per > 0 ? per : 1);
        });
        const int total = g.batch * g.kv_heads * (g.tk_pad / KBLOCK);
        cudaError_t e = launch_after_previous(sp_quant_kv_stream<D>, dim3(total < ctas ? total : ctas), dim3(256),
                                              S::DYN, st, (const uint16_t*)k, (const uint16_t*)v, buf.stats, buf.k8,
                                              buf.k_scale, buf.v8, g);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    sp_quant_kv<D><<<dim3(g.tk_pad / KBLOCK, g.kv_heads, g.batch), 256, 0, st>>>(
        (const uint16_t*)k, (const uint16_t*)v, ln, buf.stats, buf.k8, buf.k_scale, buf.v8, buf.kbias, g);
    return cudaGetLastError();
}

cudaError_t launch_prepare(int d, const void* q, const void* k, const void* v, const float* ln, const Buffers& buf,
                           const Geom& g, cudaStream_t st) {
    if (!q) return cudaErrorInvalidValue;
    return d == 64 ? prepare_d<64>(q, k, v, ln, buf, g, st) : prepare_d<128>(q, k, v, ln, buf, g, st);
}

cudaError_t launch_prepare_kv(int d, const void* k, const void* v, const float* ln, const Buffers& buf,
                              const Geom& g, cudaStream_t st) {
    return d == 64 ? prepare_d<64>(nullptr, k, v, ln, buf, g, st) : prepare_d<128>(nullptr, k, v, ln, buf, g, st);
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
    // (the partials are reduced across ranks: sp_prep does not finish them)
    sp_prep<D><<<prep_grid(g, 1), 256, 0, st>>>(
        (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, ln, buf.q8, buf.q_scale, buf.part, nullptr,
        nullptr, g, 1);
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
