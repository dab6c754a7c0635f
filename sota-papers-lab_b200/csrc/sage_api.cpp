// C ABI of libsplsage (include/splsage.h): the host side of the spl_nn::sage
// op (platform/spl-nn/src/sage/mod.rs) for sm_100a.  Validation mirrors the
// reference's checks and error texts; all GPU work is stream-ordered.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types and prototypes only: the functions are looked up at run time

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/splsage.h"
#include "sage_kernels.h"

namespace {

constexpr int QGROUP = 16, QTILE = 128, KBLOCK = 64, BLK = 128;
constexpr float FP8_MAX = 448.0f;       // mod.rs:77
constexpr float PV16_V_RANGE = 2.25f;   // mod.rs:185
constexpr int LN_Q = 1, LN_K = 2, SMOOTH_K = 4, SMOOTH_V = 8;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(SPL_SAGE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// A 3-D UINT8 tensor map {d0, d1, d2} with row pitch p1 and slab pitch p2
// (bytes), box {b0, b1, 1}, zero fill out of bounds.
int make_map(CUtensorMap* m, void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t p1, uint64_t p2,
             uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(SPL_SAGE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {p1, p2};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t elem[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, elem,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPL_SAGE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SPL_SAGE_OK;
}

// A 2-D BF16 tensor map {d0, d1} with row pitch p1 (bytes), box {b0, b1},
// 128-byte swizzle, zero fill out of bounds.
int make_map_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t d0, uint64_t d1, uint64_t p1,
                uint32_t b0, uint32_t b1) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(SPL_SAGE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {d0, d1};
    cuuint64_t strides[1] = {p1};
    cuuint32_t box[2] = {b0, b1};
    cuuint32_t elem[2] = {1, 1};
    CUresult r = enc(m, dtype, 2, const_cast<void*>(base), dims, strides, box, elem,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPL_SAGE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SPL_SAGE_OK;
}

int make_map_bf16_2d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t p1, uint32_t b0,
                     uint32_t b1) {
    return make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, d0, d1, p1, b0, b1);
}

bool fits_i32(int64_t v) { return v >= 0 && v <= 0x7fffffffLL; }

}  // namespace

struct spl_sage {
    cudaStream_t stream;
    int head_dim;
    spl_sage_config config;
    int device;
    int sm_count;
    int reserved_sms;  // SMs the persistent kernels leave free (spl_sage_reserve_sms)
    int gemm_pairs;    // GEMMs on SM pairs (spl_sage_gemm_pairs)
    uint32_t* err;     // device error word of the calls that run without a workspace
};

namespace {
// The CTA cap of a persistent kernel that leaves `reserved` SMs free (0: one
// CTA per SM).
int max_ctas(const spl_sage* s, int reserved) {
    if (reserved <= 0) return 0;
    const int n = s->sm_count - reserved;
    return n > 1 ? n : 1;
}

// ... with the engine's own reservation (spl_sage_reserve_sms).
int max_ctas(const spl_sage* s) { return max_ctas(s, s->reserved_sms); }
}  // namespace

struct spl_sage_ws {
    int head_dim;
    spl_sage_shape shape;
    spl_sage_merge merge;
    int64_t tq_pad, tk, tk_pad;
    int device;
    void* mem;
    size_t bytes;
    sp::Buffers buf;
    sp::AttnMaps maps;
    sp::Geom geom;
    bool prepared;
};

extern "C" {

const char* spl_sage_last_error(void) { return g_last_error.c_str(); }

const char* spl_sage_version(void) { return "splsage 0.1 sm_100a"; }

void spl_sage_default_config(int head_dim, spl_sage_config* out) {
    if (!out) return;
    // Tile::DEFAULT / Tile::D128 (mod.rs:128-140), FP32 PV.
    out->warps = 4;
    out->m_tiles = head_dim > 64 ? 1 : 2;
    out->stages = 3;
    out->pv_accum = SPL_SAGE_PV_F32;
}

void spl_sage_default_options(spl_sage_options* out) {
    if (!out) return;
    memset(out, 0, sizeof *out);
    out->smooth_k = 1;
    out->smooth_v = 1;
    out->qk_norm_eps = 1e-5f;
}

int spl_sage_create(void* stream, int head_dim, const spl_sage_config* cfg, spl_sage** out) {
    if (!out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_create: out is NULL");
    *out = nullptr;
    if (head_dim != 64 && head_dim != 128)
        return fail(SPL_SAGE_ERR_INVALID, "sage attention supports head dim 64 or 128, got %d", head_dim);
    spl_sage_config c;
    if (cfg)
        c = *cfg;
    else
        spl_sage_default_config(head_dim, &c);
    const uint32_t rows = 16 * c.m_tiles * c.warps;
    if (!(c.warps == 2 || c.warps == 4 || c.warps == 8) || !(c.m_tiles == 1 || c.m_tiles == 2 || c.m_tiles == 4) ||
        c.stages < 2 || c.stages > 6 || QTILE % rows != 0)
        return fail(SPL_SAGE_ERR_INVALID, "unsupported sage tile Tile { warps: %u, m_tiles: %u, stages: %u }",
                    c.warps, c.m_tiles, c.stages);
    if (c.pv_accum != SPL_SAGE_PV_F32 && c.pv_accum != SPL_SAGE_PV_F16)
        return fail(SPL_SAGE_ERR_INVALID, "unknown PV accumulation %d", c.pv_accum);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
        return fail(SPL_SAGE_ERR_DEVICE,
                    "sage attention needs an sm_100 GPU (B200: tcgen05 tensor cores, compute capability 10.0); "
                    "this GPU is %d.%d",
                    major, minor);
    uint32_t* errw = nullptr;
    e = cudaMalloc(&errw, 256);
    if (e != cudaSuccess) return cuda_fail(e, "allocate the engine's error word");
    e = cudaMemsetAsync(errw, 0, 256, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaFree(errw);
        return cuda_fail(e, "zero the engine's error word");
    }
    spl_sage* s = new spl_sage;
    s->stream = (cudaStream_t)stream;
    s->head_dim = head_dim;
    s->config = c;
    s->device = dev;
    s->sm_count = 0;
    cudaDeviceGetAttribute(&s->sm_count, cudaDevAttrMultiProcessorCount, dev);
    s->reserved_sms = 0;
    s->gemm_pairs = 1;  // measured faster at C4: bf16 1.28 -> 1.20 ms, FP8 0.81 -> 0.78 ms
    s->err = errw;
    *out = s;
    return SPL_SAGE_OK;
}

int spl_sage_reserve_sms(spl_sage* s, int n) {
    if (!s) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_reserve_sms: NULL engine");
    if (n < 0 || n >= s->sm_count)
        return fail(SPL_SAGE_ERR_INVALID, "cannot leave %d of %d SMs free", n, s->sm_count);
    s->reserved_sms = n;
    return SPL_SAGE_OK;
}

int spl_sage_gemm_pairs(spl_sage* s, int on) {
    if (!s) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_gemm_pairs: NULL engine");
    s->gemm_pairs = on ? 1 : 0;
    return SPL_SAGE_OK;
}

void spl_sage_destroy(spl_sage* s) {
    if (!s) return;
    cudaFree(s->err);
    delete s;
}

int spl_sage_plan_new(const spl_sage_shape* shape, const spl_sage_merge* merge, spl_sage_plan* out) {
    if (!shape || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_plan_new: NULL argument");
    spl_sage_shape sh = *shape;
    if (sh.kv_heads == 0) sh.kv_heads = sh.heads;
    if (sh.batch <= 0 || sh.heads <= 0 || sh.tokens <= 0 || sh.kv_heads <= 0)
        return fail(SPL_SAGE_ERR_INVALID,
                    "empty attention shape Shape { batch: %lld, heads: %lld, kv_heads: %lld, tokens: %lld }",
                    (long long)sh.batch, (long long)sh.heads, (long long)sh.kv_heads, (long long)sh.tokens);
    if (sh.heads % sh.kv_heads != 0)
        return fail(SPL_SAGE_ERR_INVALID, "heads (%lld) must be a multiple of kv_heads (%lld)", (long long)sh.heads,
                    (long long)sh.kv_heads);
    spl_sage_merge mg;
    memset(&mg, 0, sizeof mg);
    if (merge) mg = *merge;
    int64_t tk = sh.tokens;
    if (mg.stride > 1) {
        if (mg.stride != 2 && mg.stride != 4)
            return fail(SPL_SAGE_ERR_INVALID, "KV merge stride must be 2 or 4, got %d", mg.stride);
        if (mg.grid_h <= 0 || mg.grid_w <= 0)
            return fail(SPL_SAGE_ERR_INVALID, "KV merge needs a patch grid");
        if (mg.frames < 0 || mg.special < 0 || mg.dense_frames < 0)
            return fail(SPL_SAGE_ERR_INVALID, "negative frame layout field");
        const int64_t per = mg.special + mg.grid_h * mg.grid_w;
        if (mg.frames * per != sh.tokens)
            return fail(SPL_SAGE_ERR_INVALID, "frame layout covers %lld tokens, the sequence has %lld",
                        (long long)(mg.frames * per), (long long)sh.tokens);
        if (sh.causal) return fail(SPL_SAGE_ERR_INVALID, "causal attention over merged keys is not defined");
        const int64_t s_ = mg.stride;
        const int64_t merged = mg.special + ((mg.grid_h + s_ - 1) / s_) * ((mg.grid_w + s_ - 1) / s_);
        const int64_t d = mg.dense_frames < mg.frames ? mg.dense_frames : mg.frames;
        tk = d * per + (mg.frames - d) * merged;
    }
    const int64_t tq_pad = (sh.tokens + QTILE - 1) / QTILE * QTILE;
    const int64_t tk_pad = (tk + KBLOCK - 1) / KBLOCK * KBLOCK;
    if (!fits_i32(tq_pad)) return fail(SPL_SAGE_ERR_INVALID, "padded queries = %lld does not fit in i32", (long long)tq_pad);
    if (!fits_i32(tk_pad)) return fail(SPL_SAGE_ERR_INVALID, "padded keys = %lld does not fit in i32", (long long)tk_pad);
    if (!fits_i32(sh.batch * sh.heads))
        return fail(SPL_SAGE_ERR_INVALID, "batch x heads = %lld does not fit in i32", (long long)(sh.batch * sh.heads));
    if (tq_pad / 128 > 65535) return fail(SPL_SAGE_ERR_INVALID, "too many query tiles (%lld)", (long long)(tq_pad / 128));
    out->tq_pad = tq_pad;
    out->tk = tk;
    out->tk_pad = tk_pad;
    return SPL_SAGE_OK;
}

int spl_sage_workspace_create(spl_sage* s, const spl_sage_shape* shape, const spl_sage_merge* merge,
                              spl_sage_ws** out) {
    if (!s || !shape || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_workspace_create: NULL argument");
    *out = nullptr;
    spl_sage_plan plan;
    const int prc = spl_sage_plan_new(shape, merge, &plan);
    if (prc) return prc;
    spl_sage_shape sh = *shape;
    if (sh.kv_heads == 0) sh.kv_heads = sh.heads;
    spl_sage_merge mg;
    memset(&mg, 0, sizeof mg);
    if (merge) mg = *merge;
    if (mg.stride <= 1) {
        memset(&mg, 0, sizeof mg);
        mg.stride = 1;
    }
    const int64_t tq_pad = plan.tq_pad, tk = plan.tk, tk_pad = plan.tk_pad;

    const int64_t D = s->head_dim, B = sh.batch, H = sh.heads, G = sh.kv_heads;
    const int64_t q_tiles = tq_pad / QTILE;
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t n_q8 = up(B * H * tq_pad * D), n_qs = up(B * H * (tq_pad / QGROUP) * 4);
    const size_t n_k8 = up(B * G * tk_pad * D), n_ks = up(B * G * (tk_pad / KBLOCK) * 4);
    const size_t n_v8 = up(B * G * tk_pad * D), n_st = up(B * G * 4 * D * 4);
    const size_t n_kb = up(tk_pad * 4), n_part = up(B * G * q_tiles * 4 * D * 4), n_err = 256;
    const size_t n_ctl = up(B * G * 4);
    const size_t total = n_q8 + n_qs + n_k8 + n_ks + n_v8 + n_st + n_kb + n_part + n_err + n_ctl;

    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != s->device)
        return fail(SPL_SAGE_ERR_INVALID, "workspace created on device %d, the engine is on device %d", dev, s->device);
    void* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total);
    if (e != cudaSuccess) return cuda_fail(e, "allocate sage workspace");
    e = cudaMemsetAsync(mem, 0, total, s->stream);
    if (e != cudaSuccess) {
        cudaFree(mem);
        return cuda_fail(e, "zero sage workspace");
    }
    spl_sage_ws* ws = new spl_sage_ws;
    memset(ws, 0, sizeof *ws);
    ws->head_dim = (int)D;
    ws->shape = sh;
    ws->merge = mg;
    ws->tq_pad = tq_pad;
    ws->tk = tk;
    ws->tk_pad = tk_pad;
    ws->device = dev;
    ws->mem = mem;
    ws->bytes = total;
    uint8_t* p = (uint8_t*)mem;
    ws->buf.q8 = (int8_t*)p; p += n_q8;
    ws->buf.q_scale = (float*)p; p += n_qs;
    ws->buf.k8 = (int8_t*)p; p += n_k8;
    ws->buf.k_scale = (float*)p; p += n_ks;
    ws->buf.v8 = (uint8_t*)p; p += n_v8;
    ws->buf.stats = (float*)p; p += n_st;
    ws->buf.kbias = (float*)p; p += n_kb;
    ws->buf.part = (float*)p; p += n_part;
    ws->buf.err = (uint32_t*)p; p += n_err;
    ws->buf.tiles_done = (uint32_t*)p;

    const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    int rc = make_map(&ws->maps.q, ws->buf.q8, D, tq_pad, B * H, D, tq_pad * D, (uint32_t)D, 128, swz);
    if (rc == SPL_SAGE_OK)
        rc = make_map(&ws->maps.k, ws->buf.k8, D, tk_pad, B * G, D, tk_pad * D, (uint32_t)D, 128, swz);
    if (rc == SPL_SAGE_OK)
        rc = make_map(&ws->maps.v, ws->buf.v8, tk_pad, D, B * G, tk_pad, tk_pad * D, 128, (uint32_t)D,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SPL_SAGE_OK) {
        cudaFree(mem);
        delete ws;
        return rc;
    }
    *out = ws;
    return SPL_SAGE_OK;
}

void spl_sage_ws_destroy(spl_sage_ws* ws) {
    if (!ws) return;
    cudaFree(ws->mem);
    delete ws;
}

int64_t spl_sage_ws_bytes(const spl_sage_ws* ws) { return ws ? (int64_t)ws->bytes : 0; }

int spl_sage_ws_plan(const spl_sage_ws* ws, spl_sage_plan* out) {
    if (!ws || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ws_plan: NULL argument");
    out->tq_pad = ws->tq_pad;
    out->tk = ws->tk;
    out->tk_pad = ws->tk_pad;
    return SPL_SAGE_OK;
}

static int check_tensor(const char* what, const void* data, int64_t len, int64_t sb, int64_t st, int64_t sh,
                        const spl_sage_shape& shape, int64_t heads, int64_t d) {
    if (sb < 0 || st < 0 || sh < 0 || sb % 8 || st % 8 || sh % 8)
        return fail(SPL_SAGE_ERR_INVALID,
                    "%s strides must be multiples of 8 elements: Strides { batch: %lld, token: %lld, head: %lld }",
                    what, (long long)sb, (long long)st, (long long)sh);
    if (!data) return fail(SPL_SAGE_ERR_INVALID, "%s is NULL", what);
    if ((uintptr_t)data % 16)
        return fail(SPL_SAGE_ERR_INVALID, "%s must start on a multiple of 8 elements (16 bytes)", what);
    const int64_t need = (shape.batch - 1) * sb + (shape.tokens - 1) * st + (heads - 1) * sh + d;
    if (len < need)
        return fail(SPL_SAGE_ERR_INVALID, "%s holds %lld elements, its shape and strides need %lld", what,
                    (long long)len, (long long)need);
    return SPL_SAGE_OK;
}

}  // extern "C"

// The geometry of a quantiser call on ws (mod.rs:673-768): checks the
// tensors and options, then fills g; *ln receives the QK-norm parameters.
static int build_geom(spl_sage* s, const spl_sage_ws* ws, const spl_sage_tensor& q, const spl_sage_tensor& k,
                      const spl_sage_tensor& v, const spl_sage_options* opts, sp::Geom* out, const float** ln) {
    if (!s || !ws) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_prepare: NULL engine or workspace");
    if (ws->head_dim != s->head_dim)
        return fail(SPL_SAGE_ERR_INVALID, "workspace was made for head dim %d, kernels are %d", ws->head_dim,
                    s->head_dim);
    spl_sage_options o;
    if (opts)
        o = *opts;
    else
        spl_sage_default_options(&o);
    const int64_t D = s->head_dim;
    const spl_sage_shape& sh = ws->shape;
    int rc;
    // (a null Q: quantised elsewhere, by the QKV GEMM's epilogue)
    if (q.data && (rc = check_tensor("Q", q.data, q.len, q.batch, q.token, q.head, sh, sh.heads, D))) return rc;
    if ((rc = check_tensor("K", k.data, k.len, k.batch, k.token, k.head, sh, sh.kv_heads, D))) return rc;
    if ((rc = check_tensor("V", v.data, v.len, v.batch, v.token, v.head, sh, sh.kv_heads, D))) return rc;
    if (o.qk_norm_params && o.qk_norm_len < 4 * D)
        return fail(SPL_SAGE_ERR_INVALID, "QK-norm params hold %lld floats, need %lld", (long long)o.qk_norm_len,
                    (long long)(4 * D));
    int flags = 0;
    if (o.qk_norm_params) flags |= LN_Q | LN_K;
    if (o.smooth_k) flags |= SMOOTH_K;
    if (o.smooth_v) flags |= SMOOTH_V;
    // mod.rs:724-726 and :761: scale and q_mul in f32.
    const float scale = o.has_softmax_scale ? o.softmax_scale : 1.0f / sqrtf((float)D);
    const float log2e = 1.44269504088896340736f;

    sp::Geom& g = *out;
    memset(&g, 0, sizeof g);
    g.q_sb = q.batch; g.q_st = q.token; g.q_sh = q.head;
    g.k_sb = k.batch; g.k_st = k.token; g.k_sh = k.head;
    g.v_sb = v.batch; g.v_st = v.token; g.v_sh = v.head;
    g.batch = (int)sh.batch;
    g.heads = (int)sh.heads;
    g.kv_heads = (int)sh.kv_heads;
    g.tokens = (int)sh.tokens;
    g.tq_pad = (int)ws->tq_pad;
    g.tk = (int)ws->tk;
    g.tk_pad = (int)ws->tk_pad;
    g.q_tiles = (int)(ws->tq_pad / QTILE);
    const spl_sage_merge& mg = ws->merge;
    g.merge = mg.stride;
    if (mg.stride > 1) {
        const int64_t s_ = mg.stride;
        g.frames = (int)mg.frames;
        g.special = (int)mg.special;
        g.grid_h = (int)mg.grid_h;
        g.grid_w = (int)mg.grid_w;
        g.frame_tokens = (int)(mg.special + mg.grid_h * mg.grid_w);
        g.merged_frame = (int)(mg.special + ((mg.grid_h + s_ - 1) / s_) * ((mg.grid_w + s_ - 1) / s_));
        g.merged_w = (int)((mg.grid_w + s_ - 1) / s_);
        g.dense_frames = (int)(mg.dense_frames < mg.frames ? mg.dense_frames : mg.frames);
    } else {
        g.frames = 1;
    }
    g.flags = flags;
    g.causal = sh.causal ? 1 : 0;
    g.q_mul = scale * log2e;
    g.ln_eps = o.qk_norm_params ? o.qk_norm_eps : 1e-5f;
    g.v_range = s->config.pv_accum == SPL_SAGE_PV_F16 ? PV16_V_RANGE : FP8_MAX;
    *ln = o.qk_norm_params;
    return SPL_SAGE_OK;
}

extern "C" {

int spl_sage_prepare(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                     const spl_sage_options* opts) {
    sp::Geom g;
    const float* ln = nullptr;
    int rc = build_geom(s, ws, q, k, v, opts, &g, &ln);
    if (rc) return rc;
    cudaError_t e = sp::launch_prepare(s->head_dim, q.data, k.data, v.data, ln, ws->buf, g, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage prepare");
    ws->geom = g;
    ws->prepared = true;
    return SPL_SAGE_OK;
}

int spl_sage_attend(spl_sage* s, const spl_sage_ws* ws, spl_sage_tensor_mut out) {
    if (!s || !ws) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_attend: NULL engine or workspace");
    if (!ws->prepared) return fail(SPL_SAGE_ERR_STATE, "sage workspace has not been prepared");
    if (ws->head_dim != s->head_dim)
        return fail(SPL_SAGE_ERR_INVALID, "workspace was made for head dim %d, kernels are %d", ws->head_dim,
                    s->head_dim);
    int rc = check_tensor("output", out.data, out.len, out.batch, out.token, out.head, ws->shape, ws->shape.heads,
                          s->head_dim);
    if (rc) return rc;
    sp::Geom g = ws->geom;
    g.o_sb = out.batch;
    g.o_st = out.token;
    g.o_sh = out.head;
    g.max_ctas = max_ctas(s);
    cudaError_t e = sp::launch_attend(s->head_dim, ws->maps, ws->buf, g, out.data, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage attention");
    return SPL_SAGE_OK;
}

int spl_sage_forward(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                     spl_sage_tensor_mut out, const spl_sage_options* opts) {
    int rc = spl_sage_prepare(s, ws, q, k, v, opts);
    if (rc) return rc;
    return spl_sage_attend(s, ws, out);
}

int spl_sage_ws_export_reference_layout(spl_sage* s, const spl_sage_ws* ws, void* q8, float* q_scale, void* k8,
                                        float* k_scale, void* v8, float* stats, float* kbias) {
    if (!s || !ws) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ws_export_reference_layout: NULL argument");
    if (!ws->prepared) return fail(SPL_SAGE_ERR_STATE, "sage workspace has not been prepared");
    const int64_t D = ws->head_dim, B = ws->shape.batch, H = ws->shape.heads, G = ws->shape.kv_heads;
    struct {
        void* dst;
        const void* src;
        size_t n;
    } cp[] = {
        {q8, ws->buf.q8, (size_t)(B * H * ws->tq_pad * D)},
        {q_scale, ws->buf.q_scale, (size_t)(B * H * (ws->tq_pad / QGROUP) * 4)},
        {k8, ws->buf.k8, (size_t)(B * G * ws->tk_pad * D)},
        {k_scale, ws->buf.k_scale, (size_t)(B * G * (ws->tk_pad / KBLOCK) * 4)},
        {stats, ws->buf.stats, (size_t)(B * G * 4 * D * 4)},
        {kbias, ws->buf.kbias, (size_t)(ws->tk_pad * 4)},
    };
    for (auto& c : cp) {
        if (!c.dst) continue;
        cudaError_t e = cudaMemcpyAsync(c.dst, c.src, c.n, cudaMemcpyDeviceToDevice, s->stream);
        if (e != cudaSuccess) return cuda_fail(e, "export sage workspace");
    }
    if (v8) {
        cudaError_t e = sp::launch_export_v(ws->head_dim, ws->buf, ws->geom, (uint8_t*)v8, s->stream);
        if (e != cudaSuccess) return cuda_fail(e, "export sage V");
    }
    return SPL_SAGE_OK;
}

int spl_sage_status(spl_sage* s, spl_sage_ws* ws, uint32_t* device_error_word) {
    if (!s || !ws) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_status: NULL argument");
    uint32_t w = 0;
    cudaError_t e = cudaMemcpyAsync(&w, ws->buf.err, 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "read sage device status");
    if (device_error_word) *device_error_word = w;
    if (w) {
        cudaMemsetAsync(ws->buf.err, 0, 4, s->stream);
        return fail(SPL_SAGE_ERR_KERNEL, "sage kernel reported device error word 0x%08x (timeout site %u)", w,
                    (w >> 8) & 0xff);
    }
    return SPL_SAGE_OK;
}

int spl_sage_attn_resources(spl_sage* s, int* registers, int* spill_bytes) {
    if (!s || !registers || !spill_bytes) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_attn_resources: NULL argument");
    cudaError_t e = sp::attn_func_attributes(s->head_dim, 0, registers, spill_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "query attention kernel attributes");
    return SPL_SAGE_OK;
}

int spl_sage_tensor_peak(spl_sage* s, int kind, int n, int iters, double* tops, double* cycles_per_mma) {
    if (!s || !tops) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_tensor_peak: NULL argument");
    if (kind < 0 || kind > 3 || !(n == 64 || n == 128 || n == 256) || iters <= 0)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_tensor_peak: kind 0..3, n 64/128/256, iters > 0");
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, s->device);
    void* scratch = nullptr;
    cudaError_t e = cudaMalloc(&scratch, 64);
    if (e != cudaSuccess) return cuda_fail(e, "allocate peak-probe scratch");
    cudaMemsetAsync(scratch, 0, 64, s->stream);
    uint32_t* err = (uint32_t*)scratch;
    unsigned long long* cyc = (unsigned long long*)((char*)scratch + 32);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    e = sp::launch_peak(kind, n, iters, sms, err, cyc, s->stream);  // warm-up
    if (e == cudaSuccess) {
        cudaEventRecord(a, s->stream);
        e = sp::launch_peak(kind, n, iters, sms, err, cyc, s->stream);
        cudaEventRecord(b, s->stream);
    }
    float ms = 0.f;
    unsigned long long c = 0;
    uint32_t w = 0;
    if (e == cudaSuccess) e = cudaEventSynchronize(b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
    if (e == cudaSuccess) e = cudaMemcpy(&c, cyc, 8, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&w, err, 4, cudaMemcpyDeviceToHost);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFree(scratch);
    if (e != cudaSuccess) return cuda_fail(e, "tensor peak probe");
    if (w) return fail(SPL_SAGE_ERR_KERNEL, "tensor peak probe timed out (0x%08x)", w);
    const double k_elems = kind == 2 ? 16.0 : 32.0;
    const double ops = 2.0 * 128.0 * n * k_elems * 4.0 * iters * sms;
    *tops = ops / (ms * 1e-3) / 1e12;
    if (cycles_per_mma) *cycles_per_mma = (double)c / (4.0 * iters);
    return SPL_SAGE_OK;
}

int spl_sage_rope_table_1d(double base, int head_dim, int64_t positions, float* out) {
    if (!out || positions <= 0 || (head_dim != 64 && head_dim != 128) || !(base > 1.0))
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_rope_table_1d: bad arguments");
    const int pairs = head_dim / 2;
    for (int64_t t = 0; t < positions; t++)
        for (int p = 0; p < pairs; p++) {
            // RopeTable::from_angles (qkv.rs:78-96): cos / sin in f64, stored f32
            const double a = (double)t * pow(base, -(double)p / (double)pairs);
            out[(t * pairs + p) * 2] = (float)cos(a);
            out[(t * pairs + p) * 2 + 1] = (float)sin(a);
        }
    return SPL_SAGE_OK;
}

// Checks of the QKV GEMM's arguments and its geometry; kmul = the hidden
// size's required multiple.
static int qkv_setup(spl_sage* s, const spl_sage_qkv_shape* shape, const void* x, const void* w, const float* rope,
                     void* q, void* k, void* v, int kmul, sp::QkvGeom* out) {
    const spl_sage_qkv_shape& sh = *shape;
    const int64_t D = s->head_dim;
    const int64_t G = sh.kv_heads ? sh.kv_heads : sh.heads;
    const int64_t m = sh.batch * sh.tokens, n = (sh.heads + 2 * G) * D, kd = sh.hidden;
    if (sh.batch <= 0 || sh.tokens <= 0 || sh.heads <= 0 || kd <= 0)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: empty shape");
    // the epilogues route every head of a 256-channel tile to Q, K or V on
    // its own, so only the whole width must fill whole tiles
    if (n % 256 != 0)
        return fail(SPL_SAGE_ERR_INVALID,
                    "qkv: the q + k + v width (%lld channels) must be a multiple of 256 (the GEMM tile)",
                    (long long)n);
    if (kd % kmul != 0)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: hidden size %lld must be a multiple of %d", (long long)kd, kmul);
    if (!fits_i32(m) || !fits_i32(n) || !fits_i32(kd)) return fail(SPL_SAGE_ERR_INVALID, "qkv: size does not fit i32");
    if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: buffers must be 16-byte aligned");
    int half = 0;
    if (rope) {
        half = sh.rope_half;
        const bool okh = D == 64 ? (half == 16 || half == 32) : half == 64;
        if (!okh) return fail(SPL_SAGE_ERR_INVALID, "qkv: RoPE pair distance %d unsupported for head dim %lld", half,
                              (long long)D);
        if (sh.frame_len <= 0) return fail(SPL_SAGE_ERR_INVALID, "qkv: RoPE frame length is 0");
    }
    sp::QkvGeom& g = *out;
    g = sp::QkvGeom{};  // every field zero: no epilogue quantisation unless the caller sets q8
    g.m = (int)m;
    g.n = (int)n;
    g.k = (int)kd;
    g.tokens = (int)sh.tokens;
    g.hq = (int)sh.heads;
    g.hkv = (int)G;
    g.frame_len = rope ? (int)sh.frame_len : 1;
    g.rope_half = half;
    g.max_ctas = max_ctas(s);
    return SPL_SAGE_OK;
}

int spl_sage_qkv_gemm(spl_sage* s, const spl_sage_qkv_shape* shape, const void* x, const void* w, const void* bias,
                      const float* rope, void* q, void* k, void* v) {
    if (!s || !shape || !x || !w || !q || !k || !v)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_qkv_gemm: NULL argument");
    sp::QkvGeom g{};
    int rc = qkv_setup(s, shape, x, w, rope, q, k, v, 8, &g);
    if (rc) return rc;
    if (((uintptr_t)bias | (uintptr_t)rope) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: bias and RoPE table must be 16-byte aligned");
    sp::QkvMaps maps;
    const uint32_t wbox = s->gemm_pairs ? 128 : 256;  // an SM pair loads half of a 256-channel tile per CTA
    rc = make_map_bf16_2d(&maps.x, x, g.k, g.m, (uint64_t)g.k * 2, 64, 128);
    if (rc == SPL_SAGE_OK) rc = make_map_bf16_2d(&maps.w, w, g.k, g.n, (uint64_t)g.k * 2, 64, wbox);
    if (rc != SPL_SAGE_OK) return rc;
    cudaError_t e = s->gemm_pairs
                        ? sp::launch_qkv_gemm_2sm(s->head_dim, false, maps, (const uint16_t*)bias, rope, nullptr,
                                                  nullptr, (uint16_t*)q, (uint16_t*)k, (uint16_t*)v, s->err, g,
                                                  s->stream)
                        : sp::launch_qkv_gemm(s->head_dim, maps, (const uint16_t*)bias, rope, (uint16_t*)q,
                                              (uint16_t*)k, (uint16_t*)v, s->err, g, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch qkv gemm");
    return SPL_SAGE_OK;
}

int spl_sage_qkv_gemm_fp8(spl_sage* s, const spl_sage_qkv_shape* shape, const void* x8, const float* x_scale,
                          const void* w8, const float* w_scale, const void* bias, const float* rope, void* q, void* k,
                          void* v) {
    if (!s || !shape || !x8 || !x_scale || !w8 || !w_scale || !q || !k || !v)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_qkv_gemm_fp8: NULL argument");
    sp::QkvGeom g{};
    int rc = qkv_setup(s, shape, x8, w8, rope, q, k, v, 16, &g);
    if (rc) return rc;
    if (((uintptr_t)bias | (uintptr_t)rope | (uintptr_t)w_scale) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: bias, RoPE table and weight scales must be 16-byte aligned");
    sp::QkvMaps maps;
    const uint32_t wbox = s->gemm_pairs ? 128 : 256;
    rc = make_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_UINT8, x8, g.k, g.m, (uint64_t)g.k, 128, 128);
    if (rc == SPL_SAGE_OK) rc = make_map_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w8, g.k, g.n, (uint64_t)g.k, 128, wbox);
    if (rc != SPL_SAGE_OK) return rc;
    cudaError_t e = s->gemm_pairs
                        ? sp::launch_qkv_gemm_2sm(s->head_dim, true, maps, (const uint16_t*)bias, rope, x_scale,
                                                  w_scale, (uint16_t*)q, (uint16_t*)k, (uint16_t*)v, s->err, g,
                                                  s->stream)
                        : sp::launch_qkv_gemm_fp8(s->head_dim, maps, (const uint16_t*)bias, rope, x_scale, w_scale,
                                                  (uint16_t*)q, (uint16_t*)k, (uint16_t*)v, s->err, g, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch fp8 qkv gemm");
    return SPL_SAGE_OK;
}

int spl_sage_rows_fp8(spl_sage* s, const void* y, int64_t rows, int64_t c, int64_t ld, const float* tok,
                      const float* chan, const void* bias, void* q8, float* scales) {
    if (!s || !y || !q8 || !scales) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_rows_fp8: NULL argument");
    if (c != 1024 && c != 2048 && c != 3072 && c != 4096)
        return fail(SPL_SAGE_ERR_INVALID, "row_epilogue: %lld channels unsupported (1024, 2048, 3072 or 4096)",
                    (long long)c);
    if (ld < c || ld % 8 != 0)
        return fail(SPL_SAGE_ERR_INVALID, "row_epilogue: ld %lld must be a multiple of 8 and at least %lld",
                    (long long)ld, (long long)c);
    if (rows < 0 || !fits_i32(rows)) return fail(SPL_SAGE_ERR_INVALID, "row_epilogue: %lld rows", (long long)rows);
    if (((uintptr_t)y | (uintptr_t)chan | (uintptr_t)bias | (uintptr_t)q8) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "row_epilogue: buffers must be 16-byte aligned");
    if (rows == 0) return SPL_SAGE_OK;
    cudaError_t e = sp::launch_rows_fp8((const uint16_t*)y, ld, c, (int)rows, tok, chan, (const uint16_t*)bias,
                                        (uint8_t*)q8, scales, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch row_epilogue");
    return SPL_SAGE_OK;
}

int spl_sage_linear_fp8(spl_sage* s, const void* x8, const float* x_scale, const void* w8, const float* w_scale,
                        const void* bias, int64_t m, int64_t n, int64_t k, void* y) {
    if (!s || !x8 || !w8 || !y) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_linear_fp8: NULL argument");
    if ((x_scale == nullptr) != (w_scale == nullptr))
        return fail(SPL_SAGE_ERR_INVALID, "gemm: give both scales, or neither (deferred)");
    if (!x_scale && bias) return fail(SPL_SAGE_ERR_INVALID, "gemm: deferred scales leave the bias to the consumer");
    if (m <= 0 || n <= 0 || k <= 0) return fail(SPL_SAGE_ERR_INVALID, "gemm: empty shape");
    if (n % 256 != 0)
        return fail(SPL_SAGE_ERR_INVALID, "gemm: %lld output channels must be a multiple of 256 (the tile)",
                    (long long)n);
    if (k % 16 != 0) return fail(SPL_SAGE_ERR_INVALID, "gemm: k %lld must be a multiple of 16", (long long)k);
    if (!fits_i32(m) || !fits_i32(n) || !fits_i32(k)) return fail(SPL_SAGE_ERR_INVALID, "gemm: size does not fit i32");
    if (((uintptr_t)x8 | (uintptr_t)w8 | (uintptr_t)y | (uintptr_t)bias | (uintptr_t)w_scale) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "gemm: buffers must be 16-byte aligned");
    // the QKV kernel with one part of n / 128 "heads" of 128 channels and no
    // RoPE writes y row-major [m][n]
    sp::QkvGeom g{};
    memset(&g, 0, sizeof g);
    g.m = (int)m;
    g.n = (int)n;
    g.k = (int)k;
    g.tokens = (int)m;
    g.hq = (int)(n / 128);
    g.hkv = 0;
    g.frame_len = 1;
    g.rope_half = 0;
    g.max_ctas = max_ctas(s);
    sp::QkvMaps maps;
    int rc = make_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_UINT8, x8, k, m, k, 128, 128);
    if (rc == SPL_SAGE_OK)
        rc = make_map_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w8, k, n, k, 128, s->gemm_pairs ? 128 : 256);
    if (rc != SPL_SAGE_OK) return rc;
    cudaError_t e = s->gemm_pairs ? sp::launch_qkv_gemm_2sm(128, true, maps, (const uint16_t*)bias, nullptr, x_scale,
                                                            w_scale, (uint16_t*)y, nullptr, nullptr, s->err, g,
                                                            s->stream)
                                  : sp::launch_qkv_gemm_fp8(128, maps, (const uint16_t*)bias, nullptr, x_scale, w_scale,
                                                            (uint16_t*)y, nullptr, nullptr, s->err, g, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch fp8 gemm");
    return SPL_SAGE_OK;
}

int spl_sage_layer_norm_fp8(spl_sage* s, const void* x, int x_f32, int64_t rows, int64_t c, const float* gamma,
                            const float* beta, float eps, void* out, void* q8, float* scales) {
    if (!s || !x || !gamma || !beta || !q8 || !scales)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_layer_norm_fp8: NULL argument");
    if (!sp::layer_norm_width_ok(c))
        return fail(SPL_SAGE_ERR_INVALID,
                    "layer_norm: %lld channels unsupported (256, 512, 768, 1024, 1536, 2048, 3072 or 4096)",
                    (long long)c);
    if (rows < 0 || !fits_i32(rows)) return fail(SPL_SAGE_ERR_INVALID, "layer_norm: %lld rows", (long long)rows);
    if (((uintptr_t)x | (uintptr_t)gamma | (uintptr_t)beta | (uintptr_t)out | (uintptr_t)q8) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "layer_norm: buffers must be 16-byte aligned");
    if (rows == 0) return SPL_SAGE_OK;
    cudaError_t e = sp::launch_layer_norm_fp8(x, x_f32 != 0, c, gamma, beta, eps, (int)rows, (uint16_t*)out,
                                              (uint8_t*)q8, scales, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch layer_norm");
    return SPL_SAGE_OK;
}

int spl_sage_qkv_gemm_quant(spl_sage* s, spl_sage_ws* ws, const spl_sage_qkv_shape* shape, const void* x,
                            const void* w, const void* bias, const float* rope, void* q, void* k, void* v,
                            const spl_sage_options* opts) {
    if (!s || !ws || !shape) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_qkv_gemm_quant: NULL argument");
    const spl_sage_qkv_shape& sh = *shape;
    const int64_t G = sh.kv_heads ? sh.kv_heads : sh.heads;
    if (ws->shape.batch != sh.batch || ws->shape.tokens != sh.tokens || ws->shape.heads != sh.heads ||
        ws->shape.kv_heads != G)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: the workspace was made for another shape");
    const int64_t D = s->head_dim;
    spl_sage_tensor tq = {q, sh.batch * sh.tokens * sh.heads * D, sh.tokens * sh.heads * D, sh.heads * D, D};
    spl_sage_tensor tk = {k, sh.batch * sh.tokens * G * D, sh.tokens * G * D, G * D, D};
    spl_sage_tensor tv = {v, sh.batch * sh.tokens * G * D, sh.tokens * G * D, G * D, D};
    // Q quantised in the GEMM's epilogue (SM-pair kernel, dense keys, no QK
    // LayerNorm, 16-row scale groups that never straddle two sequences); the
    // quantiser then only reads K and V.  Otherwise: the GEMM, then the whole
    // quantiser on its bf16 output.
    const bool fused = s->gemm_pairs && ws->merge.stride <= 1 && !(opts && opts->qk_norm_params) &&
                       sh.tokens % QGROUP == 0;
    if (!fused) {
        if (!q) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_qkv_gemm_quant: NULL q needs the fused path");
        int rc = spl_sage_qkv_gemm(s, shape, x, w, bias, rope, q, k, v);
        if (rc) return rc;
        return spl_sage_prepare(s, ws, tq, tk, tv, opts);
    }
    if (!x || !w || !k || !v) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_qkv_gemm_quant: NULL argument");
    sp::Geom ag;
    const float* ln = nullptr;
    int rc = build_geom(s, ws, tq, tk, tv, opts, &ag, &ln);
    if (rc) return rc;
    sp::QkvGeom g{};
    if ((rc = qkv_setup(s, shape, x, w, rope, q, k, v, 8, &g))) return rc;
    if (((uintptr_t)bias | (uintptr_t)rope) % 16)
        return fail(SPL_SAGE_ERR_INVALID, "qkv: bias and RoPE table must be 16-byte aligned");
    g.q8 = ws->buf.q8;
    g.q_scale = ws->buf.q_scale;
    g.tq_pad = (int)ws->tq_pad;
    g.q_mul = ag.q_mul;
    sp::QkvMaps maps;
    rc = make_map_bf16_2d(&maps.x, x, g.k, g.m, (uint64_t)g.k * 2, 64, 128);
    if (rc == SPL_SAGE_OK) rc = make_map_bf16_2d(&maps.w, w, g.k, g.n, (uint64_t)g.k * 2, 64, 128);
    if (rc != SPL_SAGE_OK) return rc;
    cudaError_t e = sp::launch_qkv_gemm_2sm(s->head_dim, false, maps, (const uint16_t*)bias, rope, nullptr, nullptr,
                                            (uint16_t*)q, (uint16_t*)k, (uint16_t*)v, s->err, g, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch qkv gemm");
    e = sp::launch_prepare_kv(s->head_dim, k, v, ln, ws->buf, ag, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage prepare");
    ws->geom = ag;
    ws->prepared = true;
    return SPL_SAGE_OK;
}

int spl_sage_quantize_noalloc(void* stream, int head_dim, int pv_accum, const spl_sage_shape* shape,
                              spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v, const spl_sage_options* opts,
                              void* q8, float* q_scale, void* k8, float* k_scale, void* v8, float* stats) {
    // Everything this call needs besides the caller's inputs and outputs is
    // the fixed device array in sage_quant.cu: no cudaMalloc, no cudaFree.
    if (!shape || !q8 || !q_scale || !k8 || !k_scale || !v8 || !stats)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_quantize_noalloc: NULL argument");
    // The kernels store q8, k8 and v8 16 bytes at a time and the scales and
    // statistics as floats; a misaligned caller buffer would fault on the GPU.
    if ((uintptr_t)q8 % 16 || (uintptr_t)k8 % 16 || (uintptr_t)v8 % 16)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_quantize_noalloc: q8, k8 and v8 must start on 16 bytes");
    if ((uintptr_t)q_scale % 4 || (uintptr_t)k_scale % 4 || (uintptr_t)stats % 4)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_quantize_noalloc: q_scale, k_scale and stats must start on 4 bytes");
    if (head_dim != 64 && head_dim != 128)
        return fail(SPL_SAGE_ERR_INVALID, "sage attention supports head dim 64 or 128, got %d", head_dim);
    if (pv_accum != SPL_SAGE_PV_F32 && pv_accum != SPL_SAGE_PV_F16)
        return fail(SPL_SAGE_ERR_INVALID, "unknown PV accumulation %d", pv_accum);
    int dev = 0, major = 0, minor = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
        return fail(SPL_SAGE_ERR_DEVICE, "sage attention needs an sm_100 GPU; this GPU is %d.%d", major, minor);
    spl_sage_shape sh = *shape;
    if (sh.kv_heads == 0) sh.kv_heads = sh.heads;
    if (sh.batch <= 0 || sh.heads <= 0 || sh.tokens <= 0 || sh.kv_heads <= 0 || sh.heads % sh.kv_heads)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_quantize_noalloc: bad shape");
    const int64_t D = head_dim;
    const int64_t tq_pad = (sh.tokens + QTILE - 1) / QTILE * QTILE, tk_pad = (sh.tokens + KBLOCK - 1) / KBLOCK * KBLOCK;
    if (!fits_i32(tq_pad) || !fits_i32(sh.batch * sh.heads))
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_quantize_noalloc: size does not fit i32");
    const int64_t part_floats = sh.batch * sh.kv_heads * (tq_pad / QTILE) * 4 * D;
    if (part_floats > (int64_t)sp::noalloc_part_capacity())
        return fail(SPL_SAGE_ERR_INVALID,
                    "spl_sage_quantize_noalloc: batch x kv_heads x ceil(tokens/128) x 4 x head_dim = %lld floats "
                    "exceeds its fixed scratch of %lld floats; use a workspace (spl_sage_prepare)",
                    (long long)part_floats, (long long)sp::noalloc_part_capacity());
    spl_sage_options o;
    if (opts)
        o = *opts;
    else
        spl_sage_default_options(&o);
    if (o.qk_norm_params && o.qk_norm_len < 4 * D)
        return fail(SPL_SAGE_ERR_INVALID, "QK-norm params hold %lld floats, need %lld", (long long)o.qk_norm_len,
                    (long long)(4 * D));
    int rc;
    if ((rc = check_tensor("Q", q.data, q.len, q.batch, q.token, q.head, sh, sh.heads, D))) return rc;
    if ((rc = check_tensor("K", k.data, k.len, k.batch, k.token, k.head, sh, sh.kv_heads, D))) return rc;
    if ((rc = check_tensor("V", v.data, v.len, v.batch, v.token, v.head, sh, sh.kv_heads, D))) return rc;
    float* part = nullptr;
    e = sp::noalloc_part_buffer(&part);
    if (e != cudaSuccess) return cuda_fail(e, "look up the fixed quantiser scratch");

    sp::Geom g;
    memset(&g, 0, sizeof g);
    g.q_sb = q.batch; g.q_st = q.token; g.q_sh = q.head;
    g.k_sb = k.batch; g.k_st = k.token; g.k_sh = k.head;
    g.v_sb = v.batch; g.v_st = v.token; g.v_sh = v.head;
    g.batch = (int)sh.batch;
    g.heads = (int)sh.heads;
    g.kv_heads = (int)sh.kv_heads;
    g.tokens = (int)sh.tokens;
    g.tq_pad = (int)tq_pad;
    g.tk = (int)sh.tokens;
    g.tk_pad = (int)tk_pad;
    g.q_tiles = (int)(tq_pad / QTILE);
    g.merge = 1;
    g.frames = 1;
    g.flags = (o.qk_norm_params ? (LN_Q | LN_K) : 0) | (o.smooth_k ? SMOOTH_K : 0) | (o.smooth_v ? SMOOTH_V : 0);
    const float scale = o.has_softmax_scale ? o.softmax_scale : 1.0f / sqrtf((float)D);
    g.q_mul = scale * 1.44269504088896340736f;
    g.ln_eps = o.qk_norm_params ? o.qk_norm_eps : 1e-5f;
    g.v_range = pv_accum == SPL_SAGE_PV_F16 ? PV16_V_RANGE : FP8_MAX;
    sp::Buffers buf;
    memset(&buf, 0, sizeof buf);
    buf.q8 = (int8_t*)q8;
    buf.q_scale = q_scale;
    buf.k8 = (int8_t*)k8;
    buf.k_scale = k_scale;
    buf.v8 = (uint8_t*)v8;
    buf.stats = stats;
    buf.kbias = nullptr;  // dense keys: the quantiser never writes kbias
    buf.part = part;      // fully rewritten by every call before it is read
    e = sp::launch_prepare(head_dim, q.data, k.data, v.data, o.qk_norm_params, buf, g, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage quantiser");
    return SPL_SAGE_OK;
}

int spl_sage_engine_status(spl_sage* s, uint32_t* device_error_word) {
    if (!s) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_engine_status: NULL argument");
    uint32_t w = 0;
    cudaError_t e = cudaMemcpyAsync(&w, s->err, 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "read engine status");
    if (device_error_word) *device_error_word = w;
    if (w) {
        cudaMemsetAsync(s->err, 0, 4, s->stream);
        return fail(SPL_SAGE_ERR_KERNEL, "kernel reported device error word 0x%08x (timeout site %u)", w,
                    (w >> 8) & 0xff);
    }
    return SPL_SAGE_OK;
}

int spl_sage_wait_selftest(spl_sage* s, uint64_t* result) {
    if (!s || !result) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_wait_selftest: NULL argument");
    uint32_t w = 0;
    cudaError_t e = cudaMemcpyAsync(&w, s->err, 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "read engine status");
    if (w)
        return fail(SPL_SAGE_ERR_KERNEL,
                    "the engine's error word is already set (0x%08x): read it with spl_sage_engine_status first", w);
    unsigned long long* out = nullptr;
    e = cudaMalloc(&out, 4 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "allocate the wait probe's output");
    e = cudaMemsetAsync(out, 0xff, 4 * sizeof(unsigned long long), s->stream);
    if (e == cudaSuccess) e = sp::launch_wait_probe(s->err, SPL_SAGE_SELFTEST_SITE, out, s->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(result, out, 4 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    cudaFree(out);
    if (e != cudaSuccess) return cuda_fail(e, "run the wait probe");
    return SPL_SAGE_OK;
}

double spl_sage_flops(const spl_sage_ws* ws) {
    if (!ws) return 0.0;
    return 4.0 * (double)(ws->shape.batch * ws->shape.heads) * (double)ws->shape.tokens * (double)ws->tk *
           (double)ws->head_dim;
}

// ---------------------------------------------------------------- context parallelism

int spl_sage_kv_bytes(const spl_sage_ws* ws, int64_t* k8_bytes, int64_t* k_scale_bytes, int64_t* v8_bytes) {
    if (!ws) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_kv_bytes: NULL workspace");
    const int64_t B = ws->shape.batch, G = ws->shape.kv_heads, D = ws->head_dim;
    if (k8_bytes) *k8_bytes = B * G * ws->tk_pad * D;
    if (k_scale_bytes) *k_scale_bytes = B * G * (ws->tk_pad / KBLOCK) * 4;
    if (v8_bytes) *v8_bytes = B * G * ws->tk_pad * D;
    return SPL_SAGE_OK;
}

}  // extern "C"

struct spl_sage_kv {
    int head_dim;
    int64_t batch, kv_heads, tk_pad;
    int8_t* k8;
    float* k_scale;
    uint8_t* v8;
    CUtensorMap map_k, map_v;
};

extern "C" {

int spl_sage_kv_create(spl_sage* s, const spl_sage_ws* ws, void* k8, float* k_scale, void* v8, spl_sage_kv** out) {
    if (!s || !ws || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_kv_create: NULL argument");
    if (!k8 || !k_scale || !v8) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_kv_create: NULL buffer");
    if ((uintptr_t)k8 % 128 || (uintptr_t)v8 % 128 || (uintptr_t)k_scale % 16)
        return fail(SPL_SAGE_ERR_INVALID, "K/V buffers must be 128-byte aligned, k_scale 16-byte aligned");
    if (ws->head_dim != s->head_dim)
        return fail(SPL_SAGE_ERR_INVALID, "workspace was made for head dim %d, kernels are %d", ws->head_dim,
                    s->head_dim);
    if (ws->merge.stride > 1) return fail(SPL_SAGE_ERR_INVALID, "context parallelism takes dense keys only");
    const int64_t D = ws->head_dim, B = ws->shape.batch, G = ws->shape.kv_heads, T = ws->tk_pad;
    spl_sage_kv* kv = new spl_sage_kv;
    memset(kv, 0, sizeof *kv);
    kv->head_dim = (int)D;
    kv->batch = B;
    kv->kv_heads = G;
    kv->tk_pad = T;
    kv->k8 = (int8_t*)k8;
    kv->k_scale = k_scale;
    kv->v8 = (uint8_t*)v8;
    const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    int rc = make_map(&kv->map_k, k8, D, T, B * G, D, T * D, (uint32_t)D, 128, swz);
    if (rc == SPL_SAGE_OK)
        rc = make_map(&kv->map_v, v8, T, D, B * G, T, T * D, 128, (uint32_t)D, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SPL_SAGE_OK) {
        delete kv;
        return rc;
    }
    *out = kv;
    return SPL_SAGE_OK;
}

int spl_sage_kv_create_gathered(spl_sage* s, const spl_sage_ws* ws, int64_t tokens, void* k8, float* k_scale,
                                void* v8, spl_sage_kv** out) {
    if (!s || !ws || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_kv_create_gathered: NULL argument");
    if (!k8 || !k_scale || !v8) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_kv_create_gathered: NULL buffer");
    if ((uintptr_t)k8 % 128 || (uintptr_t)v8 % 128 || (uintptr_t)k_scale % 16)
        return fail(SPL_SAGE_ERR_INVALID, "K/V buffers must be 128-byte aligned, k_scale 16-byte aligned");
    if (ws->head_dim != s->head_dim)
        return fail(SPL_SAGE_ERR_INVALID, "workspace was made for head dim %d, kernels are %d", ws->head_dim,
                    s->head_dim);
    if (ws->merge.stride > 1) return fail(SPL_SAGE_ERR_INVALID, "context parallelism takes dense keys only");
    if (tokens <= 0 || tokens % BLK || !fits_i32(tokens))
        return fail(SPL_SAGE_ERR_INVALID, "gathered keys: %lld tokens must be a positive multiple of 128",
                    (long long)tokens);
    const int64_t D = ws->head_dim, B = ws->shape.batch, G = ws->shape.kv_heads, T = tokens;
    spl_sage_kv* kv = new spl_sage_kv;
    memset(kv, 0, sizeof *kv);
    kv->head_dim = (int)D;
    kv->batch = B;
    kv->kv_heads = G;
    kv->tk_pad = T;
    kv->k8 = (int8_t*)k8;
    kv->k_scale = k_scale;
    kv->v8 = (uint8_t*)v8;
    const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    int rc = make_map(&kv->map_k, k8, D, T, B * G, D, T * D, (uint32_t)D, 128, swz);
    if (rc == SPL_SAGE_OK)
        rc = make_map(&kv->map_v, v8, T, D, B * G, T, T * D, 128, (uint32_t)D, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SPL_SAGE_OK) {
        delete kv;
        return rc;
    }
    *out = kv;
    return SPL_SAGE_OK;
}

void spl_sage_kv_destroy(spl_sage_kv* kv) { delete kv; }

int spl_sage_cp_prepare(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                        const spl_sage_options* opts, float* raw) {
    if (!raw) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_prepare: NULL raw statistics buffer");
    sp::Geom g;
    const float* ln = nullptr;
    int rc = build_geom(s, ws, q, k, v, opts, &g, &ln);
    if (rc) return rc;
    if (ws->merge.stride > 1) return fail(SPL_SAGE_ERR_INVALID, "context parallelism takes dense keys only");
    cudaError_t e = sp::launch_cp_prepare(s->head_dim, q.data, k.data, v.data, ln, ws->buf, g, raw, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage context-parallel prepare");
    ws->geom = g;
    ws->prepared = false;  // K/V not quantised yet
    return SPL_SAGE_OK;
}

int spl_sage_cp_quantize_kv(spl_sage* s, spl_sage_ws* ws, spl_sage_tensor k, spl_sage_tensor v,
                            const spl_sage_options* opts, const float* raw_global, int64_t total_tokens,
                            spl_sage_kv* kv) {
    if (!raw_global || !kv) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_quantize_kv: NULL argument");
    if (total_tokens < ws->shape.tokens)
        return fail(SPL_SAGE_ERR_INVALID, "total tokens %lld is less than this rank's %lld", (long long)total_tokens,
                    (long long)ws->shape.tokens);
    if (kv->head_dim != ws->head_dim || kv->tk_pad != ws->tk_pad || kv->batch != ws->shape.batch ||
        kv->kv_heads != ws->shape.kv_heads)
        return fail(SPL_SAGE_ERR_INVALID, "the K/V buffer was made for another workspace plan");
    sp::Geom g;
    const float* ln = nullptr;
    // the query operand only has to pass the checks: K stands in for it
    spl_sage_tensor qdummy = k;
    spl_sage_ws tmp = *ws;
    tmp.shape.heads = ws->shape.kv_heads;
    int rc = build_geom(s, &tmp, qdummy, k, v, opts, &g, &ln);
    if (rc) return rc;
    g.heads = (int)ws->shape.heads;
    sp::Buffers buf = ws->buf;
    buf.k8 = kv->k8;
    buf.k_scale = kv->k_scale;
    buf.v8 = kv->v8;
    buf.kbias = nullptr;
    cudaError_t e = sp::launch_cp_quant_kv(s->head_dim, k.data, v.data, ln, buf, g, raw_global,
                                           (float)total_tokens, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage context-parallel K/V quantiser");
    ws->prepared = true;
    return SPL_SAGE_OK;
}

// One segment with `reserved` SMs left free; the engine itself is not
// changed, so other threads may use it meanwhile.
static int cp_attend(spl_sage* s, const spl_sage_ws* ws, const spl_sage_kv* kv, int64_t q_begin, int64_t q_len,
                     int64_t k_begin, int64_t k_len, int flags, float* acc, float* lse, int reserved) {
    if (!s || !ws || !kv || !acc || !lse) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_attend: NULL argument");
    if (!ws->prepared) return fail(SPL_SAGE_ERR_STATE, "sage workspace has not been prepared");
    if (kv->head_dim != ws->head_dim || kv->tk_pad != ws->tk_pad || kv->batch != ws->shape.batch ||
        kv->kv_heads != ws->shape.kv_heads)
        return fail(SPL_SAGE_ERR_INVALID, "the K/V buffer was made for another workspace plan");
    if (q_begin < 0 || q_len <= 0 || q_begin % QTILE || q_len % QTILE || q_begin + q_len > ws->tq_pad)
        return fail(SPL_SAGE_ERR_INVALID, "query segment [%lld, +%lld) must be whole 128-row tiles within %lld rows",
                    (long long)q_begin, (long long)q_len, (long long)ws->tq_pad);
    if (k_begin < 0 || k_len <= 0 || k_begin % BLK || k_begin + k_len > ws->tk)
        return fail(SPL_SAGE_ERR_INVALID, "key segment [%lld, +%lld) must start on a 128-key block within %lld keys",
                    (long long)k_begin, (long long)k_len, (long long)ws->tk);
    if (flags & ~(SPL_SAGE_CP_CAUSAL | SPL_SAGE_CP_FIRST))
        return fail(SPL_SAGE_ERR_INVALID, "unknown segment flags 0x%x", flags);
    const bool causal = (flags & SPL_SAGE_CP_CAUSAL) != 0;
    if (causal && k_len < q_len)
        return fail(SPL_SAGE_ERR_INVALID, "a causal segment needs at least as many keys as queries");
    if (q_len / QTILE > 65535) return fail(SPL_SAGE_ERR_INVALID, "too many query tiles");
    sp::Geom g = ws->geom;
    const int64_t H = ws->shape.heads, D = ws->head_dim, T = ws->shape.tokens;
    g.o_sb = T * H * D;
    g.o_st = H * D;
    g.o_sh = D;
    g.q_tile0 = (int)(q_begin / QTILE);
    g.q_tiles = (int)(q_len / QTILE);
    g.k_key0 = (int)k_begin;
    g.tk = (int)k_len;
    g.tk_pad = (int)kv->tk_pad;
    g.causal = causal ? 1 : 0;
    g.cp_first = (flags & SPL_SAGE_CP_FIRST) ? 1 : 0;
    g.max_ctas = max_ctas(s, reserved);
    g.merge = 1;
    sp::AttnMaps maps;
    maps.q = ws->maps.q;
    maps.k = kv->map_k;
    maps.v = kv->map_v;
    sp::Buffers buf = ws->buf;
    buf.k_scale = kv->k_scale;
    cudaError_t e = sp::launch_attend_partial(s->head_dim, maps, buf, g, acc, lse, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage segment attention");
    return SPL_SAGE_OK;
}

int spl_sage_cp_attend(spl_sage* s, const spl_sage_ws* ws, const spl_sage_kv* kv, int64_t q_begin, int64_t q_len,
                       int64_t k_begin, int64_t k_len, int flags, float* acc, float* lse) {
    if (!s) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_attend: NULL argument");
    return cp_attend(s, ws, kv, q_begin, q_len, k_begin, k_len, flags, acc, lse, s->reserved_sms);
}

int spl_sage_cp_attend_gathered(spl_sage* s, const spl_sage_ws* ws, const spl_sage_kv* kv_all, int64_t q_off0,
                                int64_t q_off1, spl_sage_tensor_mut out) {
    if (!s || !ws || !kv_all) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_attend_gathered: NULL argument");
    if (!ws->prepared) return fail(SPL_SAGE_ERR_STATE, "sage workspace has not been prepared");
    if (kv_all->head_dim != ws->head_dim || kv_all->batch != ws->shape.batch ||
        kv_all->kv_heads != ws->shape.kv_heads)
        return fail(SPL_SAGE_ERR_INVALID, "the gathered K/V buffer was made for another batch or kv head count");
    const int64_t T = ws->shape.tokens, C = T / 2, N = kv_all->tk_pad;
    if (T % (2 * QTILE))
        return fail(SPL_SAGE_ERR_INVALID, "this rank's %lld tokens must be two chunks of whole 128-row tiles",
                    (long long)T);
    if (q_off0 < 0 || q_off1 < 0 || q_off0 % QTILE || q_off1 % QTILE || q_off0 + C > N || q_off1 + C > N)
        return fail(SPL_SAGE_ERR_INVALID, "query chunks at %lld and %lld (of %lld rows) must be whole tiles "
                    "within the %lld gathered keys", (long long)q_off0, (long long)q_off1, (long long)C,
                    (long long)N);
    int rc = check_tensor("output", out.data, out.len, out.batch, out.token, out.head, ws->shape, ws->shape.heads,
                          s->head_dim);
    if (rc) return rc;
    sp::Geom g = ws->geom;
    g.o_sb = out.batch;
    g.o_st = out.token;
    g.o_sh = out.head;
    g.tk = (int)N;
    g.tk_pad = (int)N;
    g.causal = 1;
    g.merge = 1;
    g.q_tile0 = 0;
    g.k_key0 = 0;
    g.q_split = (int)C;
    g.q_goff0 = (int)q_off0;
    g.q_goff1 = (int)q_off1;
    g.max_ctas = max_ctas(s);
    sp::AttnMaps maps;
    maps.q = ws->maps.q;
    maps.k = kv_all->map_k;
    maps.v = kv_all->map_v;
    sp::Buffers buf = ws->buf;
    buf.k_scale = kv_all->k_scale;
    cudaError_t e = sp::launch_attend(s->head_dim, maps, buf, g, out.data, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage gathered attention");
    return SPL_SAGE_OK;
}

int spl_sage_cp_finish(spl_sage* s, const spl_sage_ws* ws, const float* acc, spl_sage_tensor_mut out) {
    if (!s || !ws || !acc) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_cp_finish: NULL argument");
    int rc = check_tensor("output", out.data, out.len, out.batch, out.token, out.head, ws->shape, ws->shape.heads,
                          s->head_dim);
    if (rc) return rc;
    sp::Geom g = ws->geom;
    g.o_sb = out.batch;
    g.o_st = out.token;
    g.o_sh = out.head;
    cudaError_t e = sp::launch_cp_finish(s->head_dim, acc, g, out.data, s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "launch sage context-parallel finish");
    return SPL_SAGE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- ring attention over NCCL

namespace {

// The NCCL functions the ring calls, looked up in the running process (a
// host that already loaded NCCL, e.g. through torch, shares its copy) or in
// libnccl.so.2; the library itself does not link NCCL.
struct NcclFns {
    decltype(&ncclAllReduce) all_reduce;
    decltype(&ncclAllGather) all_gather;
    decltype(&ncclSend) send;
    decltype(&ncclRecv) recv;
    decltype(&ncclGroupStart) group_start;
    decltype(&ncclGroupEnd) group_end;
    decltype(&ncclGetErrorString) error_string;
};

const NcclFns* nccl_fns() {
    static NcclFns f;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = RTLD_DEFAULT;
        if (!dlsym(h, "ncclSend")) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        f.all_reduce = (decltype(f.all_reduce))dlsym(h, "ncclAllReduce");
        f.all_gather = (decltype(f.all_gather))dlsym(h, "ncclAllGather");
        f.send = (decltype(f.send))dlsym(h, "ncclSend");
        f.recv = (decltype(f.recv))dlsym(h, "ncclRecv");
        f.group_start = (decltype(f.group_start))dlsym(h, "ncclGroupStart");
        f.group_end = (decltype(f.group_end))dlsym(h, "ncclGroupEnd");
        f.error_string = (decltype(f.error_string))dlsym(h, "ncclGetErrorString");
        ok = f.all_reduce && f.all_gather && f.send && f.recv && f.group_start && f.group_end && f.error_string;
    });
    return ok ? &f : nullptr;
}

int nccl_fail(const NcclFns* f, ncclResult_t r, const char* what) {
    return fail(SPL_SAGE_ERR_CUDA, "%s: %s", what, f->error_string(r));
}

}  // namespace

struct spl_sage_ring {
    int rank, world, reserved_sms;
    int64_t batch, heads, kv_heads, tokens, chunk;
    spl_sage_ws* ws;
    spl_sage_kv* kv[2];
    void* kv_mem[2];
    int64_t k8_bytes, ks_bytes, v8_bytes;
    float* acc;
    float* lse;
    float* raw;  // [bg][4][D], then raw_sum and raw_max after it
    cudaStream_t comm;
    cudaEvent_t ev_compute, ev_comm;
    // schedule 1 (gather): every rank's K/V buffer gathered (staging, world
    // x the buffer) and laid out in key order in kv_all (allocated on first use)
    int schedule;
    size_t kv_total, kso, v8o;
    void* staging;
    void* all_mem;
    spl_sage_kv* kv_all;
};

extern "C" {

void spl_sage_ring_destroy(spl_sage_ring* r) {
    if (!r) return;
    for (int i = 0; i < 2; i++) {
        spl_sage_kv_destroy(r->kv[i]);
        cudaFree(r->kv_mem[i]);
    }
    cudaFree(r->acc);
    cudaFree(r->lse);
    cudaFree(r->raw);
    spl_sage_kv_destroy(r->kv_all);
    cudaFree(r->staging);
    cudaFree(r->all_mem);
    if (r->comm) cudaStreamDestroy(r->comm);
    if (r->ev_compute) cudaEventDestroy(r->ev_compute);
    if (r->ev_comm) cudaEventDestroy(r->ev_comm);
    spl_sage_ws_destroy(r->ws);
    delete r;
}

int spl_sage_ring_create(spl_sage* s, const spl_sage_shape* local, int rank, int world, int reserved_sms,
                         spl_sage_ring** out) {
    if (!s || !local || !out) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ring_create: NULL argument");
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world)
        return fail(SPL_SAGE_ERR_INVALID, "ring: rank %d of %d ranks", rank, world);
    if (local->tokens <= 0 || local->tokens % 256)
        return fail(SPL_SAGE_ERR_INVALID,
                    "ring: each rank's %lld tokens must be two chunks of whole 128-token tiles",
                    (long long)local->tokens);
    if (reserved_sms < 0 || reserved_sms >= s->sm_count)
        return fail(SPL_SAGE_ERR_INVALID, "ring: cannot leave %d of %d SMs free", reserved_sms, s->sm_count);
    spl_sage_ring* r = new spl_sage_ring;
    memset(r, 0, sizeof *r);
    r->rank = rank;
    r->world = world;
    r->reserved_sms = world > 1 ? reserved_sms : 0;
    spl_sage_shape sh = *local;
    sh.causal = 0;
    if (sh.kv_heads == 0) sh.kv_heads = sh.heads;
    r->batch = sh.batch;
    r->heads = sh.heads;
    r->kv_heads = sh.kv_heads;
    r->tokens = sh.tokens;
    r->chunk = sh.tokens / 2;
    int rc = spl_sage_workspace_create(s, &sh, nullptr, &r->ws);
    if (rc) {
        delete r;
        return rc;
    }
    spl_sage_kv_bytes(r->ws, &r->k8_bytes, &r->ks_bytes, &r->v8_bytes);
    const int64_t D = s->head_dim;
    const size_t k8o = 0, kso = ((size_t)r->k8_bytes + 255) & ~(size_t)255;
    const size_t v8o = (kso + (size_t)r->ks_bytes + 255) & ~(size_t)255;
    const size_t kv_total = v8o + (size_t)r->v8_bytes;
    r->kv_total = kv_total;
    r->kso = kso;
    r->v8o = v8o;
    const size_t acc_n = (size_t)(r->batch * r->tokens * r->heads * D);
    const size_t lse_n = (size_t)(r->batch * r->heads * r->tokens);
    const size_t raw_n = (size_t)(r->batch * r->kv_heads * 4 * D);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaMalloc(&r->kv_mem[i], kv_total);
    if (e == cudaSuccess) e = cudaMalloc(&r->acc, acc_n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&r->lse, lse_n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&r->raw, 3 * raw_n * 4);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&r->comm, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_compute, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_comm, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        spl_sage_ring_destroy(r);
        return cuda_fail(e, "allocate the ring's buffers");
    }
    for (int i = 0; i < 2; i++) {
        uint8_t* m = (uint8_t*)r->kv_mem[i];
        rc = spl_sage_kv_create(s, r->ws, m + k8o, (float*)(m + kso), m + v8o, &r->kv[i]);
        if (rc) {
            spl_sage_ring_destroy(r);
            return rc;
        }
    }
    *out = r;
    return SPL_SAGE_OK;
}

int spl_sage_ring_schedule(spl_sage_ring* r, int schedule) {
    if (!r) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ring_schedule: NULL ring");
    if (schedule != SPL_SAGE_CP_RING && schedule != SPL_SAGE_CP_GATHER)
        return fail(SPL_SAGE_ERR_INVALID, "unknown context-parallel schedule %d", schedule);
    r->schedule = schedule;
    return SPL_SAGE_OK;
}

int spl_sage_ring_segment(int rank, int world, int step, int64_t chunk, int64_t* q_begin, int64_t* q_len,
                          int64_t* k_begin, int64_t* k_len, int* flags) {
    if (!q_begin || !q_len || !k_begin || !k_len || !flags)
        return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ring_segment: NULL argument");
    if (world < 1 || rank < 0 || rank >= world || step < 0 || step >= world || chunk <= 0)
        return fail(SPL_SAGE_ERR_INVALID, "ring: step %d of rank %d of %d ranks, chunk %lld", step, rank, world,
                    (long long)chunk);
    // the step's chunk pairs as one segment: step 0 the rank's own tokens,
    // causal, writing the accumulator; from a rank before this one both
    // query chunks against its first key chunk; from a rank after it the
    // second query chunk against both key chunks
    const int src = (rank - step + world) % world;
    *q_begin = 0;
    *q_len = 2 * chunk;
    *k_begin = 0;
    *k_len = 2 * chunk;
    *flags = 0;
    if (step == 0) {
        *flags = SPL_SAGE_CP_CAUSAL | SPL_SAGE_CP_FIRST;
    } else if (src < rank) {
        *k_len = chunk;
    } else {
        *q_begin = chunk;
        *q_len = chunk;
    }
    return SPL_SAGE_OK;
}

}  // extern "C"

// The gather schedule after step 3: every rank's K/V buffer all-gathered,
// laid out in global key order (rank s's local chunks 0 and 1 are global
// chunks s and 2P-1-s), then one causal launch over it.
static int ring_gather(spl_sage* s, spl_sage_ring* r, spl_sage_tensor_mut out, const NcclFns* nc, ncclComm_t comm) {
    const int64_t D = s->head_dim, C = r->chunk, P = r->world, T = r->tokens, N = T * P;
    const int64_t BG = r->batch * r->kv_heads;
    if (!r->kv_all) {  // first use: the whole sequence's buffer (and the staging area)
        int64_t k8b = BG * N * D, ksb = BG * (N / KBLOCK) * 4, v8b = BG * D * N;
        const size_t kso = ((size_t)k8b + 255) & ~(size_t)255, v8o = (kso + (size_t)ksb + 255) & ~(size_t)255;
        cudaError_t e = cudaMalloc(&r->all_mem, v8o + (size_t)v8b);
        if (e == cudaSuccess && P > 1) e = cudaMalloc(&r->staging, r->kv_total * (size_t)P);
        if (e != cudaSuccess) return cuda_fail(e, "allocate the gathered K/V buffers");
        uint8_t* m = (uint8_t*)r->all_mem;
        int rc = spl_sage_kv_create_gathered(s, r->ws, N, m, (float*)(m + kso), m + v8o, &r->kv_all);
        if (rc) return rc;
    }
    const uint8_t* parts = (const uint8_t*)r->kv_mem[0];
    if (P > 1) {
        ncclResult_t nr = nc->all_gather(r->kv_mem[0], r->staging, r->kv_total, ncclUint8, comm, s->stream);
        if (nr != ncclSuccess) return nccl_fail(nc, nr, "gather: K/V all-gather");
        parts = (const uint8_t*)r->staging;
    }
    // layout: k8 [bg][t][D] rows of C*D bytes, k_scale [bg][t/64] rows of
    // C/64 floats, v8 [bg][D][t] rows of C bytes
    spl_sage_kv* a = r->kv_all;
    for (int64_t src = 0; src < P; src++) {
        const uint8_t* pk = parts + (size_t)src * r->kv_total;
        for (int c = 0; c < 2; c++) {
            const int64_t gch = c == 0 ? src : 2 * P - 1 - src;
            cudaError_t e = cudaMemcpy2DAsync((uint8_t*)a->k8 + gch * C * D, (size_t)(N * D), pk + c * C * D,
                                              (size_t)(T * D), (size_t)(C * D), (size_t)BG,
                                              cudaMemcpyDeviceToDevice, s->stream);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(a->k_scale + gch * (C / KBLOCK), (size_t)(N / KBLOCK) * 4,
                                      pk + r->kso + c * (C / KBLOCK) * 4, (size_t)(T / KBLOCK) * 4,
                                      (size_t)(C / KBLOCK) * 4, (size_t)BG, cudaMemcpyDeviceToDevice, s->stream);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(a->v8 + gch * C, (size_t)N, pk + r->v8o + c * C, (size_t)T, (size_t)C,
                                      (size_t)(BG * D), cudaMemcpyDeviceToDevice, s->stream);
            if (e != cudaSuccess) return cuda_fail(e, "lay out the gathered K/V");
        }
    }
    return spl_sage_cp_attend_gathered(s, r->ws, r->kv_all, r->rank * C, (2 * P - 1 - r->rank) * C, out);
}

extern "C" {

int spl_sage_ring_forward(spl_sage* s, spl_sage_ring* r, spl_sage_tensor q, spl_sage_tensor k, spl_sage_tensor v,
                          spl_sage_tensor_mut out, const spl_sage_options* opts, void* nccl_comm) {
    if (!s || !r) return fail(SPL_SAGE_ERR_INVALID, "spl_sage_ring_forward: NULL argument");
    const NcclFns* nc = nullptr;
    if (r->world > 1) {
        if (!nccl_comm) return fail(SPL_SAGE_ERR_INVALID, "ring: %d ranks need an NCCL communicator", r->world);
        if (!(nc = nccl_fns()))
            return fail(SPL_SAGE_ERR_CUDA, "ring: NCCL is not loaded and libnccl.so.2 could not be opened");
    }
    ncclComm_t comm = (ncclComm_t)nccl_comm;
    const int64_t D = s->head_dim, C = r->chunk, P = r->world, rank = r->rank;
    const int bg = (int)(r->batch * r->kv_heads);
    const size_t raw_n = (size_t)bg * 4 * (size_t)D;
    // 1. this rank's Q quantised and its raw K/V statistics
    int rc = spl_sage_cp_prepare(s, r->ws, q, k, v, opts, r->raw);
    if (rc) return rc;
    // 2. the statistics of the whole sequence
    if (P > 1) {
        float* rsum = r->raw + raw_n;
        float* rmax = r->raw + 2 * raw_n;
        ncclResult_t nr = nc->all_reduce(r->raw, rsum, raw_n, ncclFloat32, ncclSum, comm, s->stream);
        if (nr == ncclSuccess) nr = nc->all_reduce(r->raw, rmax, raw_n, ncclFloat32, ncclMax, comm, s->stream);
        if (nr != ncclSuccess) return nccl_fail(nc, nr, "ring: statistics all-reduce");
        cudaError_t e = sp::launch_cp_merge_stats(rsum, rmax, r->raw, bg, (int)D, s->stream);
        if (e != cudaSuccess) return cuda_fail(e, "launch the statistics merge");
    }
    // 3. this rank's K/V quantised with them
    rc = spl_sage_cp_quantize_kv(s, r->ws, k, v, opts, r->raw, r->tokens * P, r->kv[0]);
    if (rc) return rc;
    if (r->schedule == SPL_SAGE_CP_GATHER) return ring_gather(s, r, out, nc, comm);
    // 4. P steps, one segment launch each, the K/V moving one rank on
    // meanwhile; the segments leave the ring's reserved SMs to NCCL
    int cur = 0;
    const int next = (int)((rank + 1) % P), prev = (int)((rank + P - 1) % P);
    for (int64_t step = 0; step < P && rc == SPL_SAGE_OK; step++) {
        const bool pass_on = step + 1 < P;
        if (pass_on) {
            // the buffer received into was read by the previous step
            cudaError_t e = cudaEventRecord(r->ev_compute, s->stream);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(r->comm, r->ev_compute, 0);
            if (e != cudaSuccess) {
                rc = cuda_fail(e, "order the ring exchange");
                break;
            }
            ncclResult_t nr = nc->group_start();
            uint8_t* snd = (uint8_t*)r->kv_mem[cur];
            uint8_t* rcv = (uint8_t*)r->kv_mem[1 - cur];
            const size_t total = ((((size_t)r->k8_bytes + 255) & ~(size_t)255) + (size_t)r->ks_bytes + 255) &
                                 ~(size_t)255;
            const size_t bytes = total + (size_t)r->v8_bytes;  // the whole buffer: k8, k_scale, v8
            if (nr == ncclSuccess) nr = nc->send(snd, bytes, ncclUint8, next, comm, r->comm);
            if (nr == ncclSuccess) nr = nc->recv(rcv, bytes, ncclUint8, prev, comm, r->comm);
            const ncclResult_t ng = nc->group_end();
            if (nr == ncclSuccess) nr = ng;
            if (nr != ncclSuccess) {
                rc = nccl_fail(nc, nr, "ring: K/V exchange");
                break;
            }
            e = cudaEventRecord(r->ev_comm, r->comm);
            if (e != cudaSuccess) {
                rc = cuda_fail(e, "record the ring exchange");
                break;
            }
        }
        int64_t qb, ql, kb, kl;
        int flags;
        rc = spl_sage_ring_segment((int)rank, (int)P, (int)step, C, &qb, &ql, &kb, &kl, &flags);
        if (rc) break;
        rc = cp_attend(s, r->ws, r->kv[cur], qb, ql, kb, kl, flags, r->acc, r->lse, r->reserved_sms);
        if (rc == SPL_SAGE_OK && pass_on) {
            cudaError_t e = cudaStreamWaitEvent(s->stream, r->ev_comm, 0);
            if (e != cudaSuccess) rc = cuda_fail(e, "wait for the ring exchange");
            cur = 1 - cur;
        }
    }
    if (rc) return rc;
    // 5. the accumulator to bf16
    return spl_sage_cp_finish(s, r->ws, r->acc, out);
}

}  // extern "C"
