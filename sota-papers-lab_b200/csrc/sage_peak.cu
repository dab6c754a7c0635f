// Tensor-core peak probes for sm_100a (the analog of the reference's
// cuda/sage_peak.cu, which measures mma.sync chains on Ada): one CTA per SM
// issues back-to-back tcgen05.mma from shared-memory operands into TMEM
// accumulators and the host times the launch.  The measured rates are the
// roofline denominators the benchmark reports beside the datasheet figures.
//
// Kinds: 0 = kind::i8 (INT8 x INT8 -> S32), 1 = kind::f8f6f4 (E4M3 x E4M3 ->
// F32), 2 = kind::f16 (BF16 x BF16 -> F32), 3 = kind::f8f6f4 (E4M3 x E4M3 ->
// F16: the accumulator SageAttention2++'s FP16 PV uses).  M = 128, N in {64, 128, 256},
// K = 32 bytes per instruction (32 8-bit / 16 16-bit elements), operands
// K-major with 128-byte swizzle; the shared memory holds zeros.
#include "sage_dev.cuh"
#include "sage_kernels.h"

namespace sp {

template <int KIND, int N>
__global__ void __launch_bounds__(128, 1) sp_peak(int iters, uint32_t* err, unsigned long long* cycles) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ uint32_t tmem_base_s;
    __shared__ __align__(8) uint64_t done;
    const uint32_t sbase = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const uint32_t sA = sbase, sB = sbase + 128 * 128;  // A: 128 rows x 128 B; B: N rows x 128 B
    for (int i = threadIdx.x; i < (128 + N) * 128 / 16; i += blockDim.x)
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(sbase + i * 16), "r"(0u));
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&done), 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc(smem_u32(&tmem_base_s), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    if (threadIdx.x == 0) {
        constexpr uint32_t IDESC = KIND == 0   ? make_idesc(C_S32, F_S8, F_S8, 128, N)
                                   : KIND == 1 ? make_idesc(C_F32, F_E4M3, F_E4M3, 128, N)
                                   : KIND == 3 ? make_idesc(C_F16, F_E4M3, F_E4M3, 128, N)
                                               : make_idesc(C_F32, F_BF16, F_BF16, 128, N);
        const unsigned long long t0 = clock64();
        for (int it = 0; it < iters; it++) {
            const uint32_t d = tmem + (uint32_t)((it & 1) * N);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t a = smem_desc(sA + kk * 32, 1024, SWZ_128B), b = smem_desc(sB + kk * 32, 1024, SWZ_128B);
                if (KIND == 0)
                    umma_i8(d, a, b, IDESC, kk > 0);
                else if (KIND == 1 || KIND == 3)
                    umma_f8(d, a, b, IDESC, kk > 0);
                else
                    umma_bf16(d, a, b, IDESC, kk > 0);
            }
        }
        tc_commit(smem_u32(&done));
        mbar_wait(smem_u32(&done), 0, err, 60, false);
        if (blockIdx.x == 0) *cycles = clock64() - t0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

template <int KIND, int N>
static cudaError_t peak_t(int iters, int sms, uint32_t* err, unsigned long long* cycles, cudaStream_t st) {
    const int smem = (128 + N) * 128 + 1024;
    cudaError_t e = cudaFuncSetAttribute(sp_peak<KIND, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    sp_peak<KIND, N><<<sms, 128, smem, st>>>(iters, err, cycles);
    return cudaGetLastError();
}

cudaError_t launch_peak(int kind, int n, int iters, int sms, uint32_t* err, unsigned long long* cycles,
                        cudaStream_t st) {
    if (kind == 0) return n == 64 ? peak_t<0, 64>(iters, sms, err, cycles, st)
                          : n == 128 ? peak_t<0, 128>(iters, sms, err, cycles, st)
                                     : peak_t<0, 256>(iters, sms, err, cycles, st);
    if (kind == 1) return n == 64 ? peak_t<1, 64>(iters, sms, err, cycles, st)
                          : n == 128 ? peak_t<1, 128>(iters, sms, err, cycles, st)
                                     : peak_t<1, 256>(iters, sms, err, cycles, st);
    if (kind == 3) return n == 64 ? peak_t<3, 64>(iters, sms, err, cycles, st)
                          : n == 128 ? peak_t<3, 128>(iters, sms, err, cycles, st)
                                     : peak_t<3, 256>(iters, sms, err, cycles, st);
    return n == 64 ? peak_t<2, 64>(iters, sms, err, cycles, st)
           : n == 128 ? peak_t<2, 128>(iters, sms, err, cycles, st)
                      : peak_t<2, 256>(iters, sms, err, cycles, st);
}

// The failure path of every bounded wait, run on purpose: warp 0 waits on an
// mbarrier that nothing arrives on and gives up after PROBE_LIMIT_NS,
// recording ERR_TIMEOUT and `site` in the error word; warp 1 waits on a
// second such barrier with the kernels' own limit and bail-out, so it leaves
// as soon as it sees the word set, as the other warps and CTAs of a failed
// launch do.  out[2w] = 1 if warp w's wait succeeded, out[2w + 1] = its
// wait in nanoseconds.  Nothing else is in flight: no TMA, no MMA, no TMEM.
constexpr unsigned long long PROBE_LIMIT_NS = 200000000ull;  // 0.2 s

__global__ void __launch_bounds__(64, 1) sp_wait_probe(uint32_t* err, uint32_t site, unsigned long long* out) {
    __shared__ __align__(8) uint64_t never[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&never[0]), 1);
        mbar_init(smem_u32(&never[1]), 1);
        fence_barrier_init();
    }
    __syncthreads();
    const unsigned long long t0 = globaltimer();
    const bool ok = warp == 0 ? mbar_wait_for<PROBE_LIMIT_NS>(smem_u32(&never[0]), 0, err, site, false)
                              : mbar_wait(smem_u32(&never[1]), 0, err, site + 1, true);
    const unsigned long long dt = globaltimer() - t0;
    if (lane == 0) {
        out[2 * warp] = ok ? 1ull : 0ull;
        out[2 * warp + 1] = dt;
    }
}

cudaError_t launch_wait_probe(uint32_t* err, uint32_t site, unsigned long long* out, cudaStream_t st) {
    sp_wait_probe<<<1, 64, 0, st>>>(err, site, out);
    return cudaGetLastError();
}

}  // namespace sp
