// Device-side helpers shared by the sm_100a kernels of libsplsage: number
// formats, mbarriers with bounded waits, TMA, tcgen05 (TMEM, UMMA) and the
// device error word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sp {

// ---------------------------------------------------------------- constants

constexpr int QGROUP = 16;   // query rows per INT8 scale (mod.rs:71)
constexpr int QTILE = 128;   // queries per quantiser tile (mod.rs:73)
constexpr int KBLOCK = 64;   // keys per K scale (mod.rs:75)
constexpr int BLK = 128;     // keys per attention block (one UMMA N)

constexpr int LN_Q = 1, LN_K = 2, SMOOTH_K = 4, SMOOTH_V = 8;

// Device error word bits (read by spl_sage_status).
constexpr uint32_t ERR_TIMEOUT = 1u << 0;       // a bounded mbarrier wait gave up
constexpr uint32_t ERR_ABORTED = 1u << 1;       // a CTA saw the error word set and left early
constexpr uint32_t ERR_SITE_SHIFT = 8;          // bits 8..15: the wait site that timed out

// A wait gives up after this many nanoseconds of %globaltimer, or after
// WAIT_MAX_TRIES unsuccessful try_waits (each one suspends for a while, so
// the count is a backstop that ends the wait even if the timer stood still).
constexpr unsigned long long WAIT_LIMIT_NS = 1500000000ull;
constexpr uint32_t WAIT_MAX_TRIES = 1u << 30;

// ---------------------------------------------------------------- formats

__device__ __forceinline__ void unpack_bf16x8(uint4 v, float* f) {
    f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
    f[4] = __uint_as_float(v.z << 16); f[5] = __uint_as_float(v.z & 0xffff0000u);
    f[6] = __uint_as_float(v.w << 16); f[7] = __uint_as_float(v.w & 0xffff0000u);
}

// bf16x2 from two floats, round to nearest even; lo in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two floats -> two E4M3 bytes (RNE, saturating at +-448); lo in the low byte.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    unsigned short r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return (uint32_t)r;
}

// Round to nearest even, clamp to the symmetric INT8 range.
__device__ __forceinline__ uint32_t s8(float x) {
    int q = __float2int_rn(x);
    q = max(-127, min(127, q));
    return (uint32_t)(q & 0xff);
}

// Four values x = v * (127 / amax) of one scale group -> four INT8 bytes, a
// in the lowest byte, each rounded to nearest even and clamped as s8 does.
// `fast` (amax zero, or finite and at least 4e-37, so that 127 / amax is
// finite): then every |x| <= 127 (1 + 2^-23), the clamp never applies, and
// the integer is read from the low mantissa bits of x + 1.5 * 2^23 (an FMA-
// pipe add and byte permutes instead of conversions).  The products must
// be rounded on their own before they come here (a plain or __fmul_rn
// product: __fadd_rn is never fused with it; a fused multiply-add, as packed
// f32x2 instructions were measured to become, breaks ties such as 63.5).
__device__ __forceinline__ uint32_t s8x4(float a, float b, float c, float d, bool fast) {
    if (!fast) return s8(a) | (s8(b) << 8) | (s8(c) << 16) | (s8(d) << 24);
    constexpr float M = 12582912.0f;
    const uint32_t ia = __float_as_uint(__fadd_rn(a, M)), ib = __float_as_uint(__fadd_rn(b, M));
    const uint32_t ic = __float_as_uint(__fadd_rn(c, M)), id = __float_as_uint(__fadd_rn(d, M));
    return __byte_perm(__byte_perm(ia, ib, 0x0040), __byte_perm(ic, id, 0x0040), 0x5410);
}

// Whether s8x4's fast path applies to a group with maximum magnitude amax.
__device__ __forceinline__ bool s8_fast(float amax) { return amax == 0.f || (amax >= 4.0e-37f && amax <= 3.0e38f); }

// Four floats -> four E4M3 bytes in one register, a in the lowest byte; the
// two halves are joined by register pairing rather than shifts.
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
    uint32_t r;
    asm("{\n .reg .b16 lo, hi;\n"
        " cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
        " cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
        " mov.b32 %0, {lo, hi};\n}"
        : "=r"(r)
        : "f"(a), "f"(b), "f"(c), "f"(d));
    return r;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------- packed f32x2 (sm_100)

__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// Element-wise max / min of two bf16x2 words; a NaN element yields the other
// element, as fmaxf / fminf do.  Exact (no rounding), so the maximum of bf16
// values taken here equals the maximum of the same values as floats.
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t bmin2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// The two bf16 halves of a word as floats (exact), lo = the low half.
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) { return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)); }

__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}


// 2^y for two arguments on the FMA pipe instead of the MUFU unit (which
// delivers only 16 results per clock per SM).  Cody-Waite style split
// y = n + f with n = rint(y) (by adding and removing the 1.5 * 2^23
// rounding constant) and f in [-0.5, 0.5]; 2^f from a degree-3 polynomial
// whose coefficients minimise the maximum relative error on [-0.5, 0.5]
// (our own Remez exchange: max relative error 7.5e-5, far below an E4M3
// step); n is added to the exponent field.  Arguments are clamped at -125 so
// the exponent never underflows past the sign bit; 2^-125 rounds to 0 in
// E4M3 anyway.
__device__ __forceinline__ void exp2_poly2(float y0, float y1, float& p0, float& p1) {
    constexpr float RND = 12582912.0f;  // 1.5 * 2^23
    constexpr float C0 = 0.99992806f, C1 = 0.69326097f, C2 = 0.24261113f, C3 = 0.05517167f;
    const uint64_t y = pk2(fmaxf(y0, -125.0f), fmaxf(y1, -125.0f));
    const uint64_t t = add2(y, pk2(RND, RND));
    const uint64_t f = sub2(y, sub2(t, pk2(RND, RND)));
    uint64_t q = fma2(f, pk2(C3, C3), pk2(C2, C2));
    q = fma2(q, f, pk2(C1, C1));
    q = fma2(q, f, pk2(C0, C0));
    float t0, t1, q0, q1;
    upk2(t, t0, t1);
    upk2(q, q0, q1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// ---------------------------------------------------------------- misc

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.u32 %0, 1, 0, P;\n}" : "=r"(pred));
    return pred;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of phase `parity` of `bar` (acquire when it returns true).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar`.  Gives up (returns false) after
// LIMIT_NS (or WAIT_MAX_TRIES), recording ERR_TIMEOUT and the wait site in
// the device error word, or, with bail_on_err, as soon as anyone has set the
// error word.  Never traps.
template <unsigned long long LIMIT_NS>
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, uint32_t* err, uint32_t site,
                                              bool bail_on_err) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (bail_on_err && ld_volatile(err) != 0) return false;
            if (globaltimer() - t0 > LIMIT_NS || i >= WAIT_MAX_TRIES) {
                atomicOr(err, ERR_TIMEOUT | ((site & 0xffu) << ERR_SITE_SHIFT));
                return false;
            }
        }
    }
}

// The kernels' wait: WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t* err, uint32_t site,
                                          bool bail_on_err = true) {
    return mbar_wait_for<WAIT_LIMIT_NS>(bar, parity, err, site, bail_on_err);
}

// All 32 lanes wait; the warp gives up together if any lane gave up.
__device__ __forceinline__ bool warp_all_wait(uint32_t bar, uint32_t parity, uint32_t* err, uint32_t site) {
    const bool ok = mbar_wait(bar, parity, err, site);
    return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, uint32_t bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05.mma this thread issued so far completes.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, INT8 x INT8 -> S32.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[smem] * B[smem]^T, FP8/FP6/FP4 kinds (E4M3 here) -> F32.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[smem] * B[smem]^T, BF16 x BF16 -> F32.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// TMEM <- shared memory, 128 lanes x 256 bits (8 columns), asynchronous,
// ordered with this thread's tcgen05.mma.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc));
}

// Instruction descriptor (tcgen05 "instruction descriptor" for kind::f16 /
// f8f6f4 / i8): c_format bits 4-5, a/b formats 7-9 / 10-12, K-major A and B
// (bits 15/16 clear), N>>3 at 17-22, M>>4 at 24-28.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt, int M, int N) {
    return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
constexpr uint32_t C_F16 = 0, C_F32 = 1, C_S32 = 2;
constexpr uint32_t F_E4M3 = 0, F_S8 = 1, F_BF16 = 1;

// Shared-memory matrix descriptor for a K-major operand tile in the
// canonical swizzled layout: rows of `row_bytes` (128 -> 128B swizzle,
// 64 -> 64B swizzle), 8-row core groups `sbo` bytes apart.  Start address
// and offsets are in 16-byte units; bits 46-47 hold the fixed version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t sbo, uint32_t swizzle_code) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3fffu);
    d |= (uint64_t)(1u) << 16;                      // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(swizzle_code & 7u) << 61;
    return d;
}
constexpr uint32_t SWZ_128B = 2, SWZ_64B = 4;

// 32 lanes x 32 bits, 32 consecutive columns: thread t of the warp gets
// row (lane base + t), columns col..col+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 16 TMEM lanes x 32 consecutive 32-bit columns, two half-warps: thread t < 16
// reads lane (base + t), columns col..col+31; thread t >= 16 reads lane
// (base + t - 16), columns col+SPLIT..col+SPLIT+31.
template <int SPLIT>
__device__ __forceinline__ void tmem_ld16x2(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], %33;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr), "n"(SPLIT));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Programmatic dependent launch.  griddep_wait: wait until the kernel this
// one was launched after (with cudaLaunchAttributeProgrammaticStreamSerialization)
// has completed and its writes are visible; without such a predecessor it
// returns at once.  griddep_launch_dependents: this CTA no longer holds back
// the start of that next kernel (which starts once every CTA of this grid
// has said so or exited; it still waits for this grid's completion before
// it reads anything this grid writes).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace sp
