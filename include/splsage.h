/*
 * libsplsage: the C ABI of the B200 (sm_100a) SageAttention2 op.
 *
 * This is the drop-in boundary for the reference's `spl_nn::sage` Rust API
 * (platform/spl-nn/src/sage/mod.rs).  Every entry point below names the
 * reference item it replaces.  Conventions, carried over from the Rust API:
 *
 *   - every call that touches the GPU enqueues on the stream given to
 *     spl_sage_create and returns without synchronising (mod.rs:509-510),
 *     except spl_sage_status, which reads a device word back;
 *   - the caller owns Q, K, V and the output (borrowed device pointers);
 *     a workspace owns the quantised tensors (mod.rs:456-495);
 *   - errors are checked before any launch and reported as a non-zero
 *     status plus a thread-local message (spl_sage_last_error), the text of
 *     the reference's `bail!` where one exists; nothing throws across the ABI;
 *   - tensors are bf16 with channels contiguous; strides are in elements and
 *     must be multiples of 8, the data pointer 16-byte aligned
 *     (Strides::check, mod.rs:251-259).
 *
 * Extensions beyond the reference (which has neither): a KV head count for
 * grouped-query attention and a causal mask.
 */
#ifndef SPLSAGE_H
#define SPLSAGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SPL_SAGE_OK 0
#define SPL_SAGE_ERR_INVALID 1     /* bad argument, shape, stride or extent */
#define SPL_SAGE_ERR_DEVICE 2      /* no usable sm_100 GPU */
#define SPL_SAGE_ERR_CUDA 3        /* a CUDA runtime / driver call failed */
#define SPL_SAGE_ERR_STATE 4       /* e.g. workspace not prepared */
#define SPL_SAGE_ERR_KERNEL 5      /* a kernel reported a device-side error (spl_sage_status) */

typedef struct spl_sage spl_sage;       /* SageAttention (mod.rs:511-520) */
typedef struct spl_sage_ws spl_sage_ws; /* Workspace (mod.rs:458-477) */

/* PvAccum (mod.rs:172-181). */
#define SPL_SAGE_PV_F32 0
#define SPL_SAGE_PV_F16 1

/* Config (mod.rs:188-201) with its Tile (mod.rs:119-124).  The tile fields
 * are validated as Tile::validate (mod.rs:158-167) does; the sm_100a kernel's
 * CTA is fixed (128 query rows per CTA, 128-key blocks), so `stages` and
 * the rest only have to be valid. */
typedef struct {
    uint32_t warps;
    uint32_t m_tiles;
    uint32_t stages;
    int32_t pv_accum; /* SPL_SAGE_PV_F32 or SPL_SAGE_PV_F16 */
} spl_sage_config;

/* Shape (mod.rs:262-268), plus kv_heads (0 = heads) and causal. */
typedef struct {
    int64_t batch;
    int64_t heads;
    int64_t kv_heads;
    int64_t tokens;
    int32_t causal;
    int32_t reserved;
} spl_sage_shape;

/* KvMerge + FrameLayout (mod.rs:273-311).  stride 0 or 1: KvMerge::Dense. */
typedef struct {
    int32_t stride;
    int32_t reserved;
    int64_t frames;
    int64_t special;
    int64_t grid_h;
    int64_t grid_w;
    int64_t dense_frames;
} spl_sage_merge;

/* Tensor / TensorMut (mod.rs:497-507) with Strides (mod.rs:203-260):
 * data + its length in bf16 elements + [batch][token][head] strides. */
typedef struct {
    const void* data;
    int64_t len;
    int64_t batch;
    int64_t token;
    int64_t head;
} spl_sage_tensor;

typedef struct {
    void* data;
    int64_t len;
    int64_t batch;
    int64_t token;
    int64_t head;
} spl_sage_tensor_mut;

/* Options (mod.rs:313-344).  qk_norm_params (device, f32 [4][head_dim]:
 * q weight, q bias, k weight, k bias) may be NULL: no QK LayerNorm. */
typedef struct {
    float softmax_scale;       /* used when has_softmax_scale */
    int32_t has_softmax_scale; /* 0: 1 / sqrt(head_dim) */
    int32_t smooth_k;          /* default 1 */
    int32_t smooth_v;          /* default 1 */
    int32_t reserved;
    const float* qk_norm_params;
    int64_t qk_norm_len; /* floats available at qk_norm_params */
    float qk_norm_eps;
    int32_t reserved2;
} spl_sage_options;

/* Plan (mod.rs:391-454). */
typedef struct {
    int64_t tq_pad; /* queries rounded up to 128 */
    int64_t tk;     /* keys after merging */
    int64_t tk_pad; /* tk rounded up to 64 */
} spl_sage_plan;

/* Config::for_head_dim (mod.rs:195-200) and Options::default (mod.rs:326-335). */
void spl_sage_default_config(int head_dim, spl_sage_config* out);
void spl_sage_default_options(spl_sage_options* out);

/* SageAttention::new / with_config (mod.rs:571-626): head_dim 64 or 128;
 * cfg NULL = spl_sage_default_config.  stream is a cudaStream_t (NULL: the
 * legacy default stream) on the current device, which must be sm_100. */
int spl_sage_create(void* stream, int head_dim, const spl_sage_config* cfg, spl_sage** out);
void spl_sage_destroy(spl_sage* s);

/* No counterpart in the reference.  The attention and QKV GEMM kernels are
 * persistent (one CTA per SM, each taking many tiles); with n > 0 they
 * launch on all but n SMs, so that kernels running beside them on other
 * streams (NCCL's send/recv during a ring step) find free SMs at once
 * instead of waiting for the whole persistent launch.  0 by default. */
int spl_sage_reserve_sms(spl_sage* s, int n);

/* No counterpart in the reference.  on = 1 (default): the QKV and FP8
 * GEMMs run on SM pairs (clusters of two CTAs, tcgen05 cta_group::2,
 * 256 x 256 tiles, each CTA loading half of both operands); 0: one SM per
 * 128 x 256 tile. */
int spl_sage_gemm_pairs(spl_sage* s, int on);

/* SageAttention::workspace (mod.rs:649-670) via Plan::new (mod.rs:405-440):
 * allocates the quantised buffers (zeroed, on the engine's stream).  merge
 * NULL = dense.  Causal with merging is rejected. */
int spl_sage_workspace_create(spl_sage* s, const spl_sage_shape* shape, const spl_sage_merge* merge,
                              spl_sage_ws** out);
void spl_sage_ws_destroy(spl_sage_ws* ws);
/* Plan::new (mod.rs:405-440): the padded query and key counts of a shape
 * and key merge, with the same checks (empty shape, merge stride 2 or 4, a
 * patch grid, a frame layout covering the sequence, i32 limits) and the
 * same error texts; merge NULL or stride <= 1 = dense.  Host only: needs no
 * engine and no GPU.  spl_sage_workspace_create applies it first. */
int spl_sage_plan_new(const spl_sage_shape* shape, const spl_sage_merge* merge, spl_sage_plan* out);
/* Workspace::bytes (mod.rs:485-494) and Workspace::plan (mod.rs:480-482). */
int64_t spl_sage_ws_bytes(const spl_sage_ws* ws);
int spl_sage_ws_plan(const spl_sage_ws* ws, spl_sage_plan* out);

/* SageAttention::prepare (mod.rs:673-836): quantise (and merge) q, k, v into
 * ws.  Three launches.  opts NULL = spl_sage_default_options. */
int spl_sage_prepare(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                     const spl_sage_options* opts);

/* SageAttention::attend (mod.rs:840-886): attention over the prepared ws,
 * bf16 into out. */
int spl_sage_attend(spl_sage* s, const spl_sage_ws* ws, spl_sage_tensor_mut out);

/* SageAttention::forward (mod.rs:889-900): prepare then attend. */
int spl_sage_forward(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                     spl_sage_tensor_mut out, const spl_sage_options* opts);

/* The quantised tensors in the reference's byte layout (the public fields
 * of Workspace, mod.rs:461-474), for the bit-exact gate: device buffers of
 *   q8 i8 [b][h][tq_pad][D], q_scale f32 [b][h][tq_pad/16],
 *   k8 i8 [b][g][tk_pad][D], k_scale f32 [b][g][tk_pad/64],
 *   v8 u8 [b][g][tk_pad/64][D][64] (E4M3, keys permuted within 16),
 *   stats f32 [b][g][4][D], kbias f32 [tk_pad]   (g = kv heads).
 * Any pointer may be NULL to skip it.  Stream-ordered copies. */
int spl_sage_ws_export_reference_layout(spl_sage* s, const spl_sage_ws* ws, void* q8, float* q_scale, void* k8,
                                        float* k_scale, void* v8, float* stats, float* kbias);

/* Reads and clears the workspace's device error word (bounded-wait
 * timeouts inside the kernels).  Synchronises the engine's stream.
 * Returns SPL_SAGE_ERR_KERNEL when the word was non-zero. */
int spl_sage_status(spl_sage* s, spl_sage_ws* ws, uint32_t* device_error_word);

/* SageAttention::attn_resources (mod.rs:641-646): registers per thread and
 * local (spill) bytes of the attention kernel. */
int spl_sage_attn_resources(spl_sage* s, int* registers, int* spill_bytes);

/* The QKV side of one transformer block: Gemm::linear_bf16 (gemm.rs:268-292,
 * y = x w^T + bias, fp32 accumulate, bf16 out) and QkvPrologue::run
 * (qkv.rs:228-301: split q | k | v, RoPE, head-major bf16) in one tcgen05
 * GEMM with a fused epilogue.  x bf16 [batch*tokens][hidden]; w bf16
 * [(heads + 2*kv_heads)*head_dim][hidden] (q rows, then k, then v); bias bf16
 * [(heads + 2*kv_heads)*head_dim] or NULL; rope NULL or f32
 * [frame_len][head_dim/2][2] (cos, sin; RopeTable, qkv.rs:65-131) applied to
 * q and k with pairs (d, d ^ rope_half) (16 or 32 at head dim 64, 64 at 128),
 * table row = token % frame_len.  Writes q bf16 [batch][tokens][heads][D],
 * k and v bf16 [batch][tokens][kv_heads][D].  The q + k + v width,
 * (heads + 2*kv_heads)*head_dim, must be a multiple of 256 channels (one
 * GEMM tile may hold heads of q, k and v); every buffer, bias and RoPE table
 * included, 16-byte aligned. */
typedef struct {
    int64_t batch;
    int64_t tokens;
    int64_t hidden;
    int64_t heads;
    int64_t kv_heads; /* 0 = heads */
    int32_t rope_half;
    int32_t frame_len;
} spl_sage_qkv_shape;

int spl_sage_qkv_gemm(spl_sage* s, const spl_sage_qkv_shape* shape, const void* x, const void* w, const void* bias,
                      const float* rope, void* q, void* k, void* v);

/* The FP8 QKV side (the reference's FP8 block,
 * apps/image-to-3d/src/vggt/trunk/block.rs:353-395): Gemm::linear_fp8 with
 * deferred weight scales (gemm.rs:294-337, y = bf16(x8 w8^T)) followed by
 * QkvPrologue::run with per-token and per-channel scales (qkv.cu:55-73:
 * y * x_scale[token] * w_scale[channel] + bias), RoPE and head-major bf16,
 * in one tcgen05 kind::f8f6f4 GEMM.  x8 E4M3 [batch*tokens][hidden] with
 * x_scale f32 [batch*tokens] (spl_sage_layer_norm_fp8 writes both); w8 E4M3
 * [(heads + 2*kv_heads)*head_dim][hidden] with w_scale f32 per output
 * channel (16-byte aligned); hidden a multiple of 16; the rest as
 * spl_sage_qkv_gemm. */
int spl_sage_qkv_gemm_fp8(spl_sage* s, const spl_sage_qkv_shape* shape, const void* x8, const float* x_scale,
                          const void* w8, const float* w_scale, const void* bias, const float* rope, void* q, void* k,
                          void* v);

/* Norm::layer_norm with Quant::PerToken (platform/spl-nn/src/norm.rs:171-274,
 * cuda/norm.cu:37-137), the LN1 that feeds the FP8 QKV GEMM: x f32 (x_f32 =
 * 1) or bf16 [rows][c], gamma and beta f32 [c]; writes q8 E4M3 [rows][c],
 * scales f32 [rows] (amax / 448, 1 for an all-zero row) and, when out is
 * not NULL, the normalised rows as bf16.  Same bytes as the reference's
 * kernel.  c = 256, 512, 768, 1024, 1536, 2048 (the reference's widths),
 * 3072 or 4096; buffers 16-byte aligned. */
int spl_sage_layer_norm_fp8(spl_sage* s, const void* x, int x_f32, int64_t rows, int64_t c, const float* gamma,
                            const float* beta, float eps, void* out, void* q8, float* scales);

/* Norm::row_epilogue with Quant::PerToken (norm.rs:280-336, cuda/norm.cu:
 * 170-229): bf16 rows y [rows][ld] (e.g. the attention output, which the
 * reference's FP8 block quantises for the proj GEMM) with optional token
 * scales tok f32 [rows], channel scales chan f32 [c] and bias bf16 [c]
 * (v = y * tok * chan + bias) to q8 E4M3 [rows][c] and scales f32 [rows]
 * (amax / 448, 1 for an all-zero row).  c = 1024, 2048, 3072 or 4096, ld a
 * multiple of 8; no activation. */
int spl_sage_rows_fp8(spl_sage* s, const void* y, int64_t rows, int64_t c, int64_t ld, const float* tok,
                      const float* chan, const void* bias, void* q8, float* scales);

/* Gemm::linear_fp8 (gemm.rs:294-337): y bf16 [m][n] = x8 [m][k] w8 [n][k]^T
 * in E4M3 on tcgen05 kind::f8f6f4 (FP32 accumulate), rounded to bf16, then,
 * with x_scale f32 [m] and w_scale f32 [n], times both scales plus bias
 * (bf16 [n] or NULL); with both scales NULL the scales are deferred to the
 * consumer (WeightScale::Deferred) and y = bf16(x8 w8^T).  n a multiple of
 * 256, k of 16. */
int spl_sage_linear_fp8(spl_sage* s, const void* x8, const float* x_scale, const void* w8, const float* w_scale,
                        const void* bias, int64_t m, int64_t n, int64_t k, void* y);

/* The block's whole QKV path up to the quantised tensors the attention
 * reads: Gemm::linear_bf16 + QkvPrologue::run + SageAttention::prepare
 * (gemm.rs:268-292, qkv.rs:228-301, mod.rs:673-836).  With the SM-pair
 * GEMMs (the default), dense keys, no QK LayerNorm and tokens a multiple of
 * 16, Q is quantised inside the GEMM's epilogue (INT8, one scale per 16
 * rows, bytes equal to spl_sage_prepare's on the bf16 Q written here) and
 * the quantiser then reads only K and V; q may then be NULL (Q is not
 * written in bf16 at all).  Otherwise spl_sage_qkv_gemm into q, k, v (bf16
 * scratch the caller owns), then spl_sage_prepare of ws from them. */
int spl_sage_qkv_gemm_quant(spl_sage* s, spl_sage_ws* ws, const spl_sage_qkv_shape* shape, const void* x,
                            const void* w, const void* bias, const float* rope, void* q, void* k, void* v,
                            const spl_sage_options* opts);

/* A 1-D RoPE table (Llama-style rotate-half, angle = t * base^(-p / (D/2))
 * for pair p) in the layout spl_sage_qkv_gemm reads, computed in f64 and
 * stored f32 like RopeTable::from_angles (qkv.rs:78-96).  Host memory,
 * positions * head_dim floats. */
int spl_sage_rope_table_1d(double base, int head_dim, int64_t positions, float* out);

/* Reads and clears the engine's own device error word (kernels launched
 * without a workspace, e.g. spl_sage_qkv_gemm).  Synchronises the stream. */
int spl_sage_engine_status(spl_sage* s, uint32_t* device_error_word);

/* The device error word: bit 0 = a bounded wait inside a kernel gave up
 * (after 1.5 s, or 2^30 tries), bit 1 = a CTA saw the word set and left
 * early, bits 8..15 = the wait site that gave up. */
#define SPL_SAGE_DEVERR_TIMEOUT 0x1u
#define SPL_SAGE_DEVERR_ABORTED 0x2u
#define SPL_SAGE_DEVERR_SITE(word) (((word) >> 8) & 0xffu)
#define SPL_SAGE_SELFTEST_SITE 99

/* Runs the failure path of the kernels' bounded waits on purpose (no
 * counterpart in the reference): one block whose warp 0 waits on an
 * mbarrier that nothing arrives on until its 0.2 s limit, recording
 * SPL_SAGE_DEVERR_TIMEOUT and site SPL_SAGE_SELFTEST_SITE in the engine's
 * error word, while warp 1 waits on another with the kernels' own limit and
 * leaves as soon as it sees the word set.  result (host, 4 values) =
 * {warp 0 succeeded, warp 0's wait in ns, warp 1 succeeded, warp 1's wait in
 * ns}.  Nothing faults and the context stays usable; the engine's word then
 * reads back through spl_sage_engine_status (which clears it).  Refuses to
 * run while the word is already set.  Synchronises the engine's stream. */
int spl_sage_wait_selftest(spl_sage* s, uint64_t* result);

/* Quantises q, k and v exactly like spl_sage_prepare (same bytes), for
 * callers that cannot allocate device memory: a library embedded in a host
 * application that owns all device memory through its own pool and forbids
 * raw cudaMalloc, or a hot path that must not take the allocator lock (or
 * risk the device synchronisation cudaMalloc and cudaFree can cause).  It
 * has no counterpart in the reference.  No engine, no workspace, and no
 * cudaMalloc, cudaFree or other allocating call: the caller passes the
 * inputs and every output, and the one piece of scratch (the per-tile
 * channel statistics) is a fixed 4 MiB device array inside the library,
 * which every GPU that loads the library keeps until the process exits.
 *   - Dense keys only (no KV merging).  Limit: batch * kv_heads *
 *     ceil(tokens / 128) * 4 * head_dim <= 1,048,576; larger calls are
 *     rejected with SPL_SAGE_ERR_INVALID (use spl_sage_prepare).
 *   - The first call on a device looks the array's device address up (and
 *     caches it with the device's current context; a device reset that
 *     re-creates the context makes the next call look it up again); make
 *     that first call before any stream capture.
 *   - q8, k8 and v8 must start on 16 bytes, q_scale, k_scale and stats on
 *     4 bytes (SPL_SAGE_ERR_INVALID otherwise): the library cannot see the
 *     outputs' sizes, so the caller sizes them as listed below.
 *   - All calls share the array and it keeps the last call's contents
 *     (each call overwrites what it reads), so calls that overlap on the
 *     GPU, on different streams, race.
 * Outputs (device buffers, the workspace's own layouts): q8 i8
 * [b][h][tq_pad][D], q_scale f32 [b][h][tq_pad/16], k8 i8 [b][g][tk_pad][D],
 * k_scale f32 [b][g][tk_pad/64], v8 u8 [b][g][D][tk_pad] (E4M3, one row per
 * channel, keys in order), stats f32 [b][g][4][D]; tq_pad = tokens rounded
 * up to 128, tk_pad to 64, g = kv heads.  Stream-ordered on `stream`. */
int spl_sage_quantize_noalloc(void* stream, int head_dim, int pv_accum, const spl_sage_shape* shape,
                              spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v, const spl_sage_options* opts,
                              void* q8, float* q_scale, void* k8, float* k_scale, void* v8, float* stats);

/* ---- Context parallelism (ring attention over GPUs) ----
 * No counterpart in the reference, which runs one sequence on one GPU.
 * Each rank holds part of a long sequence (e.g. the zig-zag chunks r and
 * 2P-1-r of 2P) in its own workspace; the host exchanges quantised K/V
 * between ranks (NCCL send/recv) and combines statistics (all-reduce):
 *   1. spl_sage_cp_prepare: quantise this rank's Q; write its raw K/V channel
 *      statistics raw f32 [b][g][4][D] = {sum K, sum V, -min V, max V}.
 *   2. combine raw over all ranks: entries 0-1 summed, 2-3 maxed.
 *   3. spl_sage_cp_quantize_kv: this rank's K/V quantised with the global
 *      statistics (total_tokens = the whole sequence) into a K/V buffer.
 *   4. for every (query chunk, key chunk) pair that is not wholly masked,
 *      spl_sage_cp_attend against the K/V buffer holding those keys
 *      (received from their owner), merged into acc / lse; pairs whose
 *      queries and keys are contiguous go in one call.
 *   5. spl_sage_cp_finish: acc to bf16.
 * The quantised K/V are not bit-identical to a single-GPU prepare (the
 * channel sums are added in another order); results are tolerance-equal. */
typedef struct spl_sage_kv spl_sage_kv; /* one rank's quantised K/V over caller memory */

/* Bytes of the three K/V buffers of ws's plan: k8 i8 [b][g][tk_pad][D],
 * k_scale f32 [b][g][tk_pad/64], v8 E4M3 [b][g][D][tk_pad]. */
int spl_sage_kv_bytes(const spl_sage_ws* ws, int64_t* k8_bytes, int64_t* k_scale_bytes, int64_t* v8_bytes);
/* TMA descriptors over caller-owned buffers (k8 and v8 128-byte aligned,
 * k_scale 16-byte aligned) of ws's plan; dense keys only. */
int spl_sage_kv_create(spl_sage* s, const spl_sage_ws* ws, void* k8, float* k_scale, void* v8, spl_sage_kv** out);
void spl_sage_kv_destroy(spl_sage_kv* kv);
int spl_sage_cp_prepare(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                        const spl_sage_options* opts, float* raw);
int spl_sage_cp_quantize_kv(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor k, spl_sage_tensor v,
                            const spl_sage_options* opts, const float* raw_global, int64_t total_tokens,
                            spl_sage_kv* kv);
/* Queries [q_begin, q_begin + q_len) of this rank (whole 128-row tiles)
 * against keys [k_begin, k_begin + k_len) of kv (k_begin a multiple of 128).
 * flags:
 *   SPL_SAGE_CP_CAUSAL  query i of the segment sees keys 0 .. i of the key
 *                       segment (the two cover the same positions);
 *                       otherwise every key is seen;
 *   SPL_SAGE_CP_FIRST   the first segment of these query rows: acc and lse
 *                       are written; otherwise the segment is merged into
 *                       them by log-sum-exp.
 * acc f32 [b][t][h][D], lse f32 [b][h][t] (t = this rank's tokens, lse the
 * log2 softmax denominator). */
#define SPL_SAGE_CP_CAUSAL 1
#define SPL_SAGE_CP_FIRST 2
int spl_sage_cp_attend(spl_sage* s, const spl_sage_ws* ws, const spl_sage_kv* kv, int64_t q_begin, int64_t q_len,
                       int64_t k_begin, int64_t k_len, int flags, float* acc, float* lse);
int spl_sage_cp_finish(spl_sage* s, const spl_sage_ws* ws, const float* acc, spl_sage_tensor_mut out);

/* Context parallelism by all-gather instead of the ring's steps (no
 * counterpart in the reference): after steps 1-3 above, the quantised K/V of
 * all ranks are gathered (e.g. ncclAllGather over NVSwitch) into one K/V
 * buffer of the whole sequence in key order, and each rank attends its two
 * query chunks to it in ONE causal launch: no per-step merge, no per-step
 * launch tail, and the zig-zag split gives every rank the same work.
 * spl_sage_kv_create_gathered: TMA descriptors over such a buffer of
 * `tokens` keys (a multiple of 128) with ws's batch, kv heads and head dim:
 * k8 i8 [b][g][tokens][D], k_scale f32 [b][g][tokens/64], v8 E4M3
 * [b][g][D][tokens] (the layouts of spl_sage_kv_bytes).
 * spl_sage_cp_attend_gathered: this rank's local query rows [0, C) sit at
 * global rows q_off0.., rows [C, 2C) at q_off1.. (C = the workspace's
 * tokens / 2, whole 128-row tiles); local row i attends the gathered keys 0
 * .. its global row; bf16 into out, with the statistics of
 * spl_sage_cp_quantize_kv. */
/* Context-parallel schedules (spl_sage_ring_schedule). */
#define SPL_SAGE_CP_RING 0   /* send/recv ring, one segment launch per step (default) */
#define SPL_SAGE_CP_GATHER 1 /* all-gather, one causal launch over the whole sequence */
int spl_sage_kv_create_gathered(spl_sage* s, const spl_sage_ws* ws, int64_t tokens, void* k8, float* k_scale,
                                void* v8, spl_sage_kv** out);
int spl_sage_cp_attend_gathered(spl_sage* s, const spl_sage_ws* ws, const spl_sage_kv* kv_all, int64_t q_off0,
                                int64_t q_off1, spl_sage_tensor_mut out);

/* The whole ring in one call, for hosts that hold their own NCCL
 * communicator (the `spl_sage_ring_forward(..., ncclComm_t, rank, world)` of
 * the drop-in boundary).  No counterpart in the reference.
 * spl_sage_ring_create: this rank's state for `local` (batch, heads,
 * kv_heads, tokens = this rank's tokens, two zig-zag chunks: chunks rank and
 * 2*world-1-rank of 2*world; a multiple of 256), its workspace, two K/V
 * buffers, the fp32 accumulator, a stream for the exchange; allocates.
 * reserved_sms: SMs the attention leaves free during the ring steps for
 * NCCL's kernel (create the communicator with ncclConfig_t.maxCTAs no larger;
 * 1 and 1 measured best on 8 B200s).
 * spl_sage_ring_forward: steps 1-5 above with the statistics all-reduced
 * (sum, max) and the K/V passed to rank + 1 over `nccl_comm` (an ncclComm_t
 * of `world` ranks, this process being `rank`; NULL when world = 1), one
 * attention launch per ring step; q, k, v and out hold this rank's tokens.
 * Stream-ordered on the engine's stream (the exchange runs on the ring's
 * own stream, ordered with it by events).  NCCL is looked up in the running
 * process, or loaded as libnccl.so.2; the library does not link it. */
typedef struct spl_sage_ring spl_sage_ring;
int spl_sage_ring_create(spl_sage* s, const spl_sage_shape* local, int rank, int world, int reserved_sms,
                         spl_sage_ring** out);
void spl_sage_ring_destroy(spl_sage_ring* r);
/* The schedule of spl_sage_ring_forward: SPL_SAGE_CP_RING (default) or
 * SPL_SAGE_CP_GATHER: after step 3 the K/V buffers of all ranks are
 * gathered with ncclAllGather into a staging area, laid out in global key
 * order by strided device copies, and attended in one causal launch per
 * rank (spl_sage_cp_attend_gathered); the whole sequence's K/V buffer and
 * the staging area are allocated by the first such forward. */
int spl_sage_ring_schedule(spl_sage_ring* r, int schedule);

/* The segment step `step` of rank `rank` attends (the schedule
 * spl_sage_ring_forward follows), as arguments of spl_sage_cp_attend with
 * chunk = each rank's tokens / 2: step 0 the rank's own two chunks, causal,
 * first of their rows; a step holding the K/V of a rank before this one both
 * query chunks against that rank's first key chunk; of a rank after it the
 * second query chunk against both key chunks.  Over the steps every
 * (query chunk, key chunk) pair of the zig-zag split with the key at or
 * before the query is attended once.  Host only. */
int spl_sage_ring_segment(int rank, int world, int step, int64_t chunk, int64_t* q_begin, int64_t* q_len,
                          int64_t* k_begin, int64_t* k_len, int* flags);
int spl_sage_ring_forward(spl_sage* s, spl_sage_ring* r, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                          spl_sage_tensor_mut out, const spl_sage_options* opts, void* nccl_comm);

/* Tensor-core peak probe (the analog of the reference's sage_peak kernels,
 * platform/spl-nn/cuda/sage_peak.cu, measured by src/sage/tests.rs:758-794):
 * one CTA per SM issues `iters` x 4 back-to-back tcgen05.mma of M=128, N=n
 * (64, 128 or 256), 32 bytes of K, kind 0 = i8 -> s32, 1 = f8f6f4 e4m3 -> f32,
 * 2 = f16 (bf16) -> f32, 3 = f8f6f4 e4m3 -> f16 (the FP16 PV accumulator of
 * SageAttention2++, PvAccum::F16).  Returns the rate over all SMs in tera-ops/s and the
 * cycles per instruction of SM 0.  Synchronises the engine's stream. */
int spl_sage_tensor_peak(spl_sage* s, int kind, int n, int iters, double* tops, double* cycles_per_mma);

/* flops (mod.rs:905-910): 4 * B * H * Tq * Tk * D of the workspace's plan. */
double spl_sage_flops(const spl_sage_ws* ws);

/* The last error message of this thread ("" when none). */
const char* spl_sage_last_error(void);

/* Library version string. */
const char* spl_sage_version(void);

#ifdef __cplusplus
}
#endif
#endif
