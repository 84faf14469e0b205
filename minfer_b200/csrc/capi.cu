// libmfcuda: C ABI over the sm_100a kernels (see include/minfer_cuda.h).
//
// The manager part replaces the reference's Metal context
// (src/interfaces/metal_interface.mm): a process-global table of ranks, each
// with its device, one stream, pinned step record and the captured CUDA graphs
// of its frames. Ops launch with programmatic dependent launch so a kernel's
// weight prefetch overlaps its predecessor's tail, inside captured graphs too.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cstddef>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <set>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemv_inst.cuh"
#include "gemv_tma.cuh"
#include "minfer_cuda.h"
#include "misc.cuh"

struct mf_buf {
    void* ptr;
    size_t bytes;
    int rank;
};

// One tensor-parallel rank's exchange state (see comm.cuh).
struct mf_comm {
    int rank = 0;         // manager rank (device) this comm lives on
    char* region = nullptr;
    std::vector<void*> opened;  // peers' regions mapped through CUDA IPC
    mf::CommDev dev = {};
    mf::CommLayout layout = {};
    bool connected = false;
};

namespace mf {
const void* attn_kernel_ptr(int group, int kv_dtype);
}

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

#define MF_CK(expr)                                                                              \
    do {                                                                                         \
        cudaError_t e_ = (expr);                                                                 \
        if (e_ != cudaSuccess) return fail(MF_E_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

#define MF_REQUIRE(cond, code, ...)                 \
    do {                                            \
        if (!(cond)) return fail(code, __VA_ARGS__); \
    } while (0)

struct Rank {
    int device = 0;
    cudaStream_t stream = nullptr;
    int32_t* h_step = nullptr;  // pinned step record (MF_STEP_RECORD_BYTES)
    void* d_step = nullptr;
    std::map<int, cudaGraphExec_t> frames;
    cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
    int recording = -1;  // frame id being captured
    int pending = -1;    // frame id to launch at end_frame
    // pinned staging ring for large host -> device copies (weights from the model file's mapping)
    void* stage[4] = {};
    cudaEvent_t stage_ev[4] = {};
    bool stage_ready = false;
    std::shared_ptr<std::mutex> stage_mu = std::make_shared<std::mutex>();
};

struct Ctx {
    bool inited = false;
    std::vector<Rank> ranks;
    std::set<mf_buf*> bufs;
};

Ctx g;

bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = std::getenv("MF_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

int num_sms() {
    static int n[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (n[dev] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n[dev] = v > 0 ? v : 148;
    }
    return n[dev];
}

cudaStream_t resolve(void* s) {
    if (s) return (cudaStream_t)s;
    int dev = 0;
    cudaGetDevice(&dev);
    for (auto& r : g.ranks)
        if (r.device == dev) return r.stream;
    return (cudaStream_t)0;
}

// Launch-shape knobs for tuning sweeps (defaults are the tuned values):
// MF_GEMV_CTAS_PER_SM caps resident GEMV CTAs per SM (0 = occupancy limit),
// MF_GEMV_PF_TILES sets the L2 prefetch depth in tiles.
int env_int(const char* name, int dflt) {
    const char* e = std::getenv(name);
    return (e && *e) ? std::atoi(e) : dflt;
}

// Optional uniform shared-memory carveout for every kernel of the token loop
// (MF_CARVEOUT=percent): consecutive kernels then never make an SM drain to
// reconfigure L1/shared. Off by default (measured slower on B200).
void set_carveout_once(const void* fn) {
    static const int carveout = env_int("MF_CARVEOUT", -1);  // -1: driver default, else percent
    if (carveout < 0) return;
    static std::set<std::pair<int, const void*>> done;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (done.insert({dev, fn}).second)
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
}

// Launch with the programmatic-serialization attribute.
cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    set_carveout_once(fn);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Launch as clusters of `cluster` CTAs along x, with the programmatic-serialization attribute.
cudaError_t launch_cluster(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args,
                           int cluster) {
    set_carveout_once(fn);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Per-kernel one-time attribute setup + occupancy cache.
struct KInfo {
    int max_smem_set = 0;
    std::map<size_t, int> occ;
};
std::map<std::pair<int, const void*>, KInfo> g_kinfo;
std::mutex g_kmu;

int prepare(const void* fn, int threads, size_t smem, int* blocks_per_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_kmu);
    KInfo& ki = g_kinfo[{dev, fn}];
    // opt in to large dynamic shared memory (static + dynamic above 48 KB)
    if ((int)smem > ki.max_smem_set && smem >= 32 * 1024) {
        MF_CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        ki.max_smem_set = (int)smem;
    }
    auto it = ki.occ.find(smem);
    if (it == ki.occ.end()) {
        int b = 0;
        MF_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, threads, smem));
        it = ki.occ.emplace(smem, b).first;
    }
    *blocks_per_sm = it->second;
    MF_REQUIRE(it->second > 0, MF_E_UNSUPPORTED, "kernel does not fit on an SM (smem %zu B)", smem);
    return MF_OK;
}

const void* gemv_ptr(int dtype, int xm, int ym, int T, int R) {
    if (xm == mf::X_AR_NORM || ym == mf::Y_PUSH || ym == mf::Y_MOE_PUSH) {
        switch (dtype) {
            case MF_F32: return mf::gemv_tp_kernel_ptr_f32(xm, ym, T, R);
            case MF_F16: return mf::gemv_tp_kernel_ptr_f16(xm, ym, T, R);
            case MF_BF16: return mf::gemv_tp_kernel_ptr_bf16(xm, ym, T, R);
            default: return nullptr;
        }
    }
    switch (dtype) {
        case MF_F32: return mf::gemv_kernel_ptr_f32(xm, ym, T, R);
        case MF_F16: return mf::gemv_kernel_ptr_f16(xm, ym, T, R);
        case MF_BF16: return mf::gemv_kernel_ptr_bf16(xm, ym, T, R);
        default: return nullptr;
    }
}

int vec_of(int dtype) { return dtype == MF_F32 ? 4 : 8; }
size_t esz_of(int dtype) { return dtype == MF_F32 ? 4 : 2; }

// Pick (T, R): the fewest idle lanes over K, then more threads, then taller tiles.
void choose_shape(int K, int dtype, int ym, int* T_out, int* R_out) {
    const int vec = vec_of(dtype);
    const int Ts[3] = {256, 128, 64};
    const int Rs[3] = {8, 4, 2};
    double best = 1e30;
    int bT = 256, bR = 8;
    for (int ti = 0; ti < 3; ++ti) {
        for (int ri = 0; ri < 3; ++ri) {
            const int T = Ts[ti], R = Rs[ri], PC = 8 / R;
            if ((ym == mf::Y_MOE_DOWN || ym == mf::Y_MOE_PUSH) && R != 8) continue;
            const long long step = (long long)PC * T * vec;
            const long long nsteps = (K + step - 1) / step;
            const double waste = (double)(nsteps * step) / K;
            // prefer exact fits; among equals more threads, then R=4 (balanced)
            const double score = waste * 1000.0 - T * 0.01 - (R == 4 ? 0.001 : 0.0);
            if (score < best) {
                best = score;
                bT = T;
                bR = R;
            }
        }
    }
    *T_out = bT;
    *R_out = bR;
}

// The manager step record's decode-status field on the current device (the
// TMA-fed kernels report a wait that gave up there).
int* decode_status_ptr() {
    int dev = 0;
    cudaGetDevice(&dev);
    for (auto& r : g.ranks)
        if (r.device == dev) return (int*)r.d_step + MF_STEP_DSTATUS;
    return nullptr;
}

const void* gemv_tma_fn(int dtype, int xm, int ym, int nwc, int j) {
    switch (dtype) {
        case MF_F32: return mf::gemv_tma_ptr_f32(xm, ym, nwc, j);
        case MF_F16: return mf::gemv_tma_ptr_f16(xm, ym, nwc, j);
        case MF_BF16: return mf::gemv_tma_ptr_bf16(xm, ym, nwc, j);
        default: return nullptr;
    }
}

// The TMA-fed dense GEMV (gemv_tma.cuh) for the plain and normalised store,
// residual and SwiGLU forms: 1 when it launched, 0 when the shape is left to
// the register-fed kernel (MF_GEMV_TMA=0 sends everything there), < 0 on error.
int try_gemv_tma(int dtype, int xm, int ym, const mf::GemvParams& q, cudaStream_t st) {
    static const int on = env_int("MF_GEMV_TMA", 1);
    static const long long timeout_ms = env_int("MF_DECODE_TIMEOUT_MS", 1000);
    // ring geometry and CTAs per SM (MF_GEMV_TMA_STAGE_KB / _RING_KB / _CPS: tuning knobs)
    static const size_t stage_target = (size_t)env_int("MF_GEMV_TMA_STAGE_KB", mf::GT_STAGE_TARGET / 1024) * 1024;
    static const size_t ring_bytes = (size_t)env_int("MF_GEMV_TMA_RING_KB", mf::GT_RING_BYTES / 1024) * 1024;
    static const int cps = std::max(1, env_int("MF_GEMV_TMA_CPS", 2));
    // rows up to 10 KB (K <= 5120 in bf16) run whole; wider rows of the plain
    // store/residual forms are split over a cluster of CTAs (split-K, slices
    // of at most 8 KB, reduced in distributed shared memory); MF_GEMV_TMA_SPLIT=0
    // leaves those to the register-fed kernel
    static const int max_row_kb = env_int("MF_GEMV_TMA_MAX_ROW_KB", 10);
    static const int split_on = env_int("MF_GEMV_TMA_SPLIT", 1);
    static const int tp_on = env_int("MF_GEMV_TMA_TP", 1);  // the tensor-parallel receive/send forms
    static const int moe_on = env_int("MF_GEMV_TMA_MOE", 1);  // the grouped-expert gate/up form
    if (!on) return 0;
    const bool tp = xm == mf::X_AR_NORM || ym == mf::Y_PUSH;
    if (tp && !tp_on) return 0;
    if (!(xm == mf::X_PLAIN || xm == mf::X_NORM || xm == mf::X_AR_NORM) ||
        !(ym == mf::Y_STORE || ym == mf::Y_RESID || ym == mf::Y_SWIGLU || ym == mf::Y_PUSH))
        return 0;
    if (q.counter || q.gather_logits) return 0;
    // grouped experts: the SwiGLU form over every selected expert stored here
    const bool grouped = q.expert_ids != nullptr;
    if (grouped && !(moe_on && xm == mf::X_NORM && ym == mf::Y_SWIGLU && q.rows_per_expert > 0 &&
                     q.rows_per_expert % 2 == 0 && q.rows % q.rows_per_expert == 0 &&
                     q.rows / q.rows_per_expert <= 32))
        return 0;
    const int vec = vec_of(dtype);
    const size_t esz = esz_of(dtype);
    const size_t full_row = (size_t)q.K * esz;
    if (grouped && full_row > (size_t)max_row_kb * 1024) return 0;
    int ks = 1;
    if (full_row > (size_t)max_row_kb * 1024) {
        if (!split_on || xm != mf::X_PLAIN || ym == mf::Y_SWIGLU) return 0;
        for (int s = 2; s <= 8 && ks == 1; ++s)
            if (q.K % s == 0 && (q.K / s) % (2 * vec) == 0 && (size_t)(q.K / s) * esz <= 8 * 1024) ks = s;
        if (ks == 1) return 0;
    }
    const int Ks = q.K / ks;  // columns of this kernel's rows (a slice when split)
    const int NV = Ks / vec;
    int nwc = 8, j = (NV + 8 * 32 - 1) / (8 * 32);
    if (j > 8) {
        nwc = 16;
        j = (NV + 16 * 32 - 1) / (16 * 32);
        if (j > 8) return 0;
        j = 8;
    } else {
        static const int js[] = {1, 2, 3, 4, 6, 8};
        for (int c : js)
            if (c >= j) {
                j = c;
                break;
            }
    }
    const void* fn = gemv_tma_fn(dtype, xm, ym, nwc, j);
    if (!fn) return 0;
    const int RU = ym == mf::Y_SWIGLU ? 2 : 1;
    const size_t row_bytes = (size_t)Ks * esz;
    int rps = (int)(stage_target / row_bytes) / RU * RU;
    if (rps < RU) rps = RU;
    const size_t stage_bytes = (size_t)rps * row_bytes;
    if (stage_bytes > 2 * stage_target && stage_bytes > 2 * (size_t)mf::GT_STAGE_TARGET) return 0;
    int stages = (int)(ring_bytes / stage_bytes);
    stages = std::max(2, std::min(stages, mf::GT_MAX_STAGES));
    const long long units = q.rows / RU;
    int* status = decode_status_ptr();
    if (!status) return 0;
    // CTAs per SM: `cps` (one with 16 consumer warps), fewer when the
    // occupancy calculation says they do not fit; the grid is one wave (all
    // CTAs resident at once, which the all-reduce receive's grid barrier needs)
    int want = nwc == 16 ? 1 : cps;
    long long nblk = 1;
    size_t smem = 0;
    for (int attempt = 0;; ++attempt) {
        nblk = std::max<long long>(1, std::min<long long>((long long)num_sms() * want / ks, units));
        const size_t max_rows = (size_t)((units + nblk - 1) / nblk) * RU;
        smem = (size_t)stages * stage_bytes + max_rows * nwc * sizeof(float);
        if (smem > 200 * 1024) return 0;
        int bps = 0;
        int rc = prepare(fn, (nwc + 1) * 32, smem, &bps);
        if (rc) return rc;
        if (bps >= want) break;
        if (bps < 1 || attempt > 0) return 0;
        want = bps;
    }
    mf::GemvTmaParams p = {};
    p.w = (const char*)q.w + q.w_offset * esz;
    p.row_bytes = row_bytes;
    p.rows = q.rows;
    p.K = Ks;
    p.x = q.x;
    p.nw = q.nw;
    p.eps = q.eps;
    p.y = q.y;
    p.rows_per_stage = rps;
    p.stages = stages;
    p.stage_bytes = (uint32_t)stage_bytes;
    p.status = status;
    p.timeout_ns = (unsigned long long)std::max(1ll, timeout_ms) * 1000000ull;
    p.ksplit = ks;
    p.row_stride = full_row;
    if (tp) {
        p.comm = q.comm;
        p.ar_seq = q.ar_seq;
        p.step = q.step;
        p.x_res = q.x_res;
        p.x_out = q.x_out;
        if (xm == mf::X_AR_NORM) p.x = q.x_out;  // read after the receive and the grid barrier
    }
    if (grouped) {
        p.expert_ids = q.expert_ids;
        p.rows_per_expert = q.rows_per_expert;
        p.expert_bytes = (unsigned long long)q.rows_per_expert * row_bytes;
        p.ep_lo = q.ep_lo;
        p.ep_n = q.ep_n;
    }
    void* args[] = {&p};
    if (ks == 1) MF_CK(launch(fn, dim3((unsigned)nblk), dim3((nwc + 1) * 32), smem, st, args));
    else MF_CK(launch_cluster(fn, dim3((unsigned)(nblk * ks)), dim3((nwc + 1) * 32), smem, st, args, ks));
    return 1;
}

// The TMA-fed grouped expert down projection (moe_down_tma_kernel): 1 when it
// launched, 0 when left to the register-fed kernel (MF_GEMV_TMA_MOE=0, expert
// parallelism, rows wider than 10 KB or K beyond 8 vectors per lane), < 0 on error.
int try_moe_down_tma(int dtype, const mf::GemvParams& q, cudaStream_t st, bool ids_early, bool push = false) {
    static const int on = env_int("MF_GEMV_TMA", 1) && env_int("MF_GEMV_TMA_MOE", 1);
    static const long long timeout_ms = env_int("MF_DECODE_TIMEOUT_MS", 1000);
    static const size_t stage_target = (size_t)env_int("MF_MOE_TMA_STAGE_KB", 16) * 1024;
    static const size_t ring_bytes = (size_t)env_int("MF_GEMV_TMA_RING_KB", mf::GT_RING_BYTES / 1024) * 1024;
    if (!on || q.n_slots < 1 || q.n_slots > mf::MD_WARPS) return 0;
    const int vec = vec_of(dtype);
    const size_t row_bytes = (size_t)q.K * esz_of(dtype);
    if (row_bytes > 10 * 1024 || row_bytes % 16 != 0) return 0;
    const int NV = q.K / vec;
    int j = (NV + 31) / 32;
    static const int js[] = {1, 2, 3, 4, 6, 8};
    int jj = 0;
    for (int c : js)
        if (c >= j) {
            jj = c;
            break;
        }
    if (!jj) return 0;
    const void* fn = dtype == MF_F32   ? mf::moe_down_tma_ptr_f32(jj)
                     : dtype == MF_F16 ? mf::moe_down_tma_ptr_f16(jj)
                                       : mf::moe_down_tma_ptr_bf16(jj);
    if (!fn) return 0;
    const size_t slot_bytes = (size_t)q.n_slots * row_bytes;  // one output row of every slot
    int R = (int)std::max<size_t>(1, stage_target / slot_bytes);
    const size_t stage_bytes = (size_t)R * slot_bytes;
    int stages = (int)std::max<size_t>(2, std::min<size_t>(ring_bytes / stage_bytes, mf::GT_MAX_STAGES));
    int* status = decode_status_ptr();
    if (!status) return 0;
    const long long nblk = std::max<long long>(1, std::min<long long>((long long)num_sms() * 2, q.rows));
    const size_t max_rows = (size_t)((q.rows + nblk - 1) / nblk);
    const size_t smem = (size_t)stages * stage_bytes + max_rows * q.n_slots * sizeof(float);
    if (smem > 200 * 1024) return 0;
    int bps = 0;
    int rc = prepare(fn, (mf::MD_WARPS + 1) * 32, smem, &bps);
    if (rc) return rc;
    if (bps < 1) return 0;
    mf::MoeDownTmaParams p = {};
    p.w = (const char*)q.w + q.w_offset * esz_of(dtype);
    p.row_bytes = row_bytes;
    p.expert_bytes = (unsigned long long)q.rows_per_expert * row_bytes;
    p.rows = q.rows;
    p.K = q.K;
    p.k = q.n_slots;
    p.h = q.x;
    p.ids = q.expert_ids;
    p.ew = q.expert_w;
    p.x = q.y;
    p.rows_per_stage = R;
    p.stages = stages;
    p.stage_bytes = (uint32_t)stage_bytes;
    p.status = status;
    p.timeout_ns = (unsigned long long)std::max(1ll, timeout_ms) * 1000000ull;
    p.ids_early = ids_early ? 1 : 0;
    p.ep_lo = q.ep_lo;
    p.ep_n = q.ep_n;
    if (push) {
        p.push = 1;
        p.comm = q.comm;
        p.ar_seq = q.ar_seq;
        p.step = q.step;
    }
    void* args[] = {&p};
    MF_CK(launch(fn, dim3((unsigned)nblk), dim3((mf::MD_WARPS + 1) * 32), smem, st, args));
    return 1;
}

int run_gemv(int dtype, int xm, int ym, mf::GemvParams& p, long long units, cudaStream_t st, int max_grid = 0) {
    static const int cps_cap = env_int("MF_GEMV_CTAS_PER_SM", 0);
    static const int pf_tiles = env_int("MF_GEMV_PF_TILES", 1);
    p.pf_tiles = pf_tiles;
    MF_REQUIRE(p.K > 0 && p.K % 16 == 0, MF_E_INVALID, "d_in must be a positive multiple of 16 (got %d)", p.K);
    MF_REQUIRE(p.rows > 0, MF_E_INVALID, "d_out must be positive");
    MF_REQUIRE(((uintptr_t)p.w + p.w_offset * esz_of(dtype)) % 16 == 0, MF_E_INVALID,
               "weight rows must start 16-byte aligned");
    MF_REQUIRE(((uintptr_t)p.x) % 16 == 0, MF_E_INVALID, "activation vector must be 16-byte aligned");
    if (max_grid == 0) {
        const int tr = try_gemv_tma(dtype, xm, ym, p, st);
        if (tr < 0) return tr;
        if (tr == 1) return MF_OK;
    }
    int T, R;
    choose_shape(p.K, dtype, ym, &T, &R);
    const void* fn = gemv_ptr(dtype, xm, ym, T, R);
    MF_REQUIRE(fn != nullptr, MF_E_UNSUPPORTED, "no GEMV kernel for dtype %d", dtype);
    // X_NORM keeps the norm weights beside x
    const bool norm = xm == mf::X_NORM || xm == mf::X_AR_NORM;
    const bool moe_down = ym == mf::Y_MOE_DOWN || ym == mf::Y_MOE_PUSH;
    const size_t xfloats = moe_down ? (size_t)p.K * p.n_slots : (size_t)p.K * (norm ? 2 : 1);
    const size_t smem = xfloats * sizeof(float);
    MF_REQUIRE(smem <= 200 * 1024, MF_E_UNSUPPORTED, "activation vector of %zu floats exceeds shared memory", xfloats);
    int bps = 0;
    int rc = prepare(fn, T, smem, &bps);
    if (rc) return rc;
    if (cps_cap > 0 && bps > cps_cap) bps = cps_cap;
    long long grid = (long long)num_sms() * bps;
    if (grid > units) grid = units;
    if (max_grid > 0 && grid > max_grid) grid = max_grid;
    if (grid < 1) grid = 1;
    void* args[] = {&p};
    MF_CK(launch(fn, dim3((unsigned)grid), dim3(T), smem, st, args));
    return MF_OK;
}

bool valid_dtype(int dt) { return dt == MF_F32 || dt == MF_F16 || dt == MF_BF16; }

constexpr int LMH_MAX_GRID = 4096;

}  // namespace

namespace mf {
// Used by entry points compiled in other files of this library.
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }
cudaStream_t resolve_stream(void* stream) { return resolve(stream); }
}  // namespace mf

extern "C" {

// ===================================================================== manager

int mf_last_error(char* buf, size_t n) {
    if (!buf || n == 0) return MF_E_INVALID;
    std::snprintf(buf, n, "%s", g_err);
    return MF_OK;
}

int mf_device_count(int* count) {
    MF_REQUIRE(count, MF_E_INVALID, "null count");
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) {
        *count = 0;
        return fail(MF_E_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = c;
    return MF_OK;
}

int mf_init(int n_ranks, const int* devices) {
    MF_REQUIRE(n_ranks >= 1 && n_ranks <= 64, MF_E_INVALID, "n_ranks out of range: %d", n_ranks);
    if (g.inited) {
        bool same = (int)g.ranks.size() == n_ranks;
        for (int i = 0; same && i < n_ranks; ++i) same = g.ranks[i].device == (devices ? devices[i] : i);
        MF_REQUIRE(same, MF_E_STATE, "mf_init called again with different ranks; call mf_shutdown first");
        return MF_OK;
    }
    int ndev = 0;
    MF_CK(cudaGetDeviceCount(&ndev));
    g.ranks.assign(n_ranks, Rank{});
    for (int i = 0; i < n_ranks; ++i) {
        Rank& r = g.ranks[i];
        r.device = devices ? devices[i] : i;
        MF_REQUIRE(r.device >= 0 && r.device < ndev, MF_E_INVALID, "device %d not present (%d visible)", r.device,
                   ndev);
        MF_CK(cudaSetDevice(r.device));
        MF_CK(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking));
        MF_CK(cudaHostAlloc((void**)&r.h_step, MF_STEP_RECORD_BYTES, cudaHostAllocDefault));
        std::memset(r.h_step, 0, MF_STEP_RECORD_BYTES);
        MF_CK(cudaMalloc(&r.d_step, MF_STEP_RECORD_BYTES));
        MF_CK(cudaMemset(r.d_step, 0, MF_STEP_RECORD_BYTES));
    }
    MF_CK(cudaSetDevice(g.ranks[0].device));
    g.inited = true;
    return MF_OK;
}

int mf_shutdown(void) {
    if (!g.inited) return MF_OK;
    for (auto& r : g.ranks) {
        cudaSetDevice(r.device);
        if (r.stream) cudaStreamSynchronize(r.stream);
        for (auto& kv : r.frames) cudaGraphExecDestroy(kv.second);
        r.frames.clear();
        if (r.ev_start) cudaEventDestroy(r.ev_start);
        if (r.ev_stop) cudaEventDestroy(r.ev_stop);
        if (r.stream) cudaStreamDestroy(r.stream);
        if (r.h_step) cudaFreeHost(r.h_step);
        if (r.d_step) cudaFree(r.d_step);
        for (int i = 0; i < 4; ++i) {
            if (r.stage[i]) cudaFreeHost(r.stage[i]);
            if (r.stage_ev[i]) cudaEventDestroy(r.stage_ev[i]);
        }
    }
    for (mf_buf* b : g.bufs) {
        cudaSetDevice(g.ranks[b->rank].device);
        cudaFree(b->ptr);
        delete b;
    }
    g.bufs.clear();
    g.ranks.clear();
    g.inited = false;
    return MF_OK;
}

static int alloc_impl(size_t bytes, int rank, mf_buf** out) {
    MF_REQUIRE(g.inited, MF_E_STATE, "mf_init not called");
    MF_REQUIRE(out, MF_E_INVALID, "null out");
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    MF_REQUIRE(bytes > 0, MF_E_INVALID, "zero-byte buffer");
    MF_CK(cudaSetDevice(g.ranks[rank].device));
    size_t free_b = 0, total_b = 0;
    MF_CK(cudaMemGetInfo(&free_b, &total_b));
    MF_REQUIRE(bytes <= free_b, MF_E_OOM, "buffer of %zu bytes exceeds free device memory (%zu)", bytes, free_b);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(MF_E_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    mf_buf* b = new mf_buf{p, bytes, rank};
    g.bufs.insert(b);
    *out = b;
    return MF_OK;
}

int mf_alloc(size_t bytes, int rank, mf_buf** out) {
    int rc = alloc_impl(bytes, rank, out);
    if (rc) return rc;
    MF_CK(cudaMemsetAsync((*out)->ptr, 0, bytes, g.ranks[rank].stream));
    MF_CK(cudaStreamSynchronize(g.ranks[rank].stream));
    return MF_OK;
}

// Host -> device copy of a large pageable range (typically a tensor inside the
// model file's mapping) through a ring of pinned staging buffers: host threads
// fill one buffer while the copy engine drains the previous ones, so reading
// the mapping and the PCIe transfer overlap. Small copies go directly.
constexpr size_t STAGE_BYTES = 32u << 20;
constexpr int STAGE_SLOTS = 4;
constexpr int STAGE_THREADS = 4;
constexpr size_t STAGE_MIN = 8u << 20;

static void parallel_memcpy(char* dst, const char* src, size_t n) {
    const size_t part = (n + STAGE_THREADS - 1) / STAGE_THREADS;
    std::thread th[STAGE_THREADS - 1];
    int nt = 0;
    for (int t = 1; t < STAGE_THREADS; ++t) {
        const size_t o = (size_t)t * part;
        if (o >= n) break;
        const size_t len = std::min(part, n - o);
        th[nt++] = std::thread([=] { std::memcpy(dst + o, src + o, len); });
    }
    std::memcpy(dst, src, std::min(part, n));
    for (int t = 0; t < nt; ++t) th[t].join();
}

static int h2d(Rank& r, char* dst, const char* src, size_t bytes) {
    if (bytes >= STAGE_MIN) {
        std::lock_guard<std::mutex> lk(*r.stage_mu);
        if (!r.stage_ready) {
            bool ok = true;
            for (int i = 0; i < STAGE_SLOTS && ok; ++i)
                ok = cudaHostAlloc(&r.stage[i], STAGE_BYTES, cudaHostAllocPortable) == cudaSuccess &&
                     cudaEventCreateWithFlags(&r.stage_ev[i], cudaEventDisableTiming) == cudaSuccess;
            if (!ok) {
                cudaGetLastError();
                for (int i = 0; i < STAGE_SLOTS; ++i) {
                    if (r.stage[i]) cudaFreeHost(r.stage[i]);
                    if (r.stage_ev[i]) cudaEventDestroy(r.stage_ev[i]);
                    r.stage[i] = nullptr;
                    r.stage_ev[i] = nullptr;
                }
            }
            r.stage_ready = ok;
        }
        if (r.stage_ready) {
            size_t off = 0;
            for (int k = 0; off < bytes; ++k) {
                const size_t n = std::min(STAGE_BYTES, bytes - off);
                const int slot = k % STAGE_SLOTS;
                MF_CK(cudaEventSynchronize(r.stage_ev[slot]));  // this buffer's previous copy is done
                parallel_memcpy((char*)r.stage[slot], src + off, n);
                MF_CK(cudaMemcpyAsync(dst + off, r.stage[slot], n, cudaMemcpyHostToDevice, r.stream));
                MF_CK(cudaEventRecord(r.stage_ev[slot], r.stream));
                off += n;
            }
            MF_CK(cudaStreamSynchronize(r.stream));
            return MF_OK;
        }
    }
    MF_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, r.stream));
    MF_CK(cudaStreamSynchronize(r.stream));
    return MF_OK;
}

int mf_upload(const void* host, size_t bytes, int rank, mf_buf** out) {
    MF_REQUIRE(host, MF_E_INVALID, "null host pointer");
    int rc = alloc_impl(bytes, rank, out);
    if (rc) return rc;
    rc = h2d(g.ranks[rank], (char*)(*out)->ptr, (const char*)host, bytes);
    if (rc) {  // the caller gets no buffer on failure: release it here
        mf_release(*out);
        *out = nullptr;
    }
    return rc;
}

void mf_release(mf_buf* buf) {
    if (!buf || !g.bufs.count(buf)) return;
    cudaSetDevice(g.ranks[buf->rank].device);
    cudaStreamSynchronize(g.ranks[buf->rank].stream);
    cudaFree(buf->ptr);
    g.bufs.erase(buf);
    delete buf;
}

void* mf_ptr(const mf_buf* buf) { return buf ? buf->ptr : nullptr; }
size_t mf_size(const mf_buf* buf) { return buf ? buf->bytes : 0; }

int mf_read(const mf_buf* buf, size_t offset, void* host, size_t bytes) {
    MF_REQUIRE(buf && host, MF_E_INVALID, "null argument");
    MF_REQUIRE(offset + bytes <= buf->bytes, MF_E_INVALID, "read past the end of the buffer");
    Rank& r = g.ranks[buf->rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaMemcpyAsync(host, (char*)buf->ptr + offset, bytes, cudaMemcpyDeviceToHost, r.stream));
    MF_CK(cudaStreamSynchronize(r.stream));
    return MF_OK;
}

int mf_write(mf_buf* buf, size_t offset, const void* host, size_t bytes) {
    MF_REQUIRE(buf && host, MF_E_INVALID, "null argument");
    MF_REQUIRE(offset + bytes <= buf->bytes, MF_E_INVALID, "write past the end of the buffer");
    Rank& r = g.ranks[buf->rank];
    MF_CK(cudaSetDevice(r.device));
    return h2d(r, (char*)buf->ptr + offset, (const char*)host, bytes);
}

int mf_write_2d(mf_buf* buf, size_t offset, size_t dst_pitch, const void* host, size_t src_pitch, size_t width,
                size_t rows) {
    MF_REQUIRE(buf && host, MF_E_INVALID, "null argument");
    MF_REQUIRE(width <= dst_pitch && width <= src_pitch, MF_E_INVALID, "width exceeds pitch");
    MF_REQUIRE(rows == 0 || offset + (rows - 1) * dst_pitch + width <= buf->bytes, MF_E_INVALID,
               "2-D write past the end of the buffer");
    if (rows == 0 || width == 0) return MF_OK;
    Rank& r = g.ranks[buf->rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaMemcpy2DAsync((char*)buf->ptr + offset, dst_pitch, host, src_pitch, width, rows,
                            cudaMemcpyHostToDevice, r.stream));
    MF_CK(cudaStreamSynchronize(r.stream));
    return MF_OK;
}

int mf_copy(mf_buf* dst, size_t dst_off, const mf_buf* src, size_t src_off, size_t bytes) {
    MF_REQUIRE(dst && src, MF_E_INVALID, "null argument");
    MF_REQUIRE(dst->rank == src->rank, MF_E_INVALID, "copy across ranks");
    MF_REQUIRE(dst_off + bytes <= dst->bytes && src_off + bytes <= src->bytes, MF_E_INVALID, "copy out of bounds");
    Rank& r = g.ranks[dst->rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaMemcpyAsync((char*)dst->ptr + dst_off, (const char*)src->ptr + src_off, bytes,
                          cudaMemcpyDeviceToDevice, r.stream));
    MF_CK(cudaStreamSynchronize(r.stream));
    return MF_OK;
}

int mf_host_alloc(size_t bytes, void** out) {
    MF_REQUIRE(out && bytes > 0, MF_E_INVALID, "bad arguments");
    MF_CK(cudaHostAlloc(out, bytes, cudaHostAllocDefault));
    return MF_OK;
}

void mf_host_free(void* p) {
    if (p) cudaFreeHost(p);
}

int mf_copy_to_host_async(void* host, const void* dev, size_t bytes, void* stream) {
    MF_REQUIRE(host && dev, MF_E_INVALID, "null argument");
    MF_CK(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, resolve(stream)));
    return MF_OK;
}

void* mf_stream(int rank) {
    if (rank < 0 || rank >= (int)g.ranks.size()) return nullptr;
    return (void*)g.ranks[rank].stream;
}

int mf_step_state(int rank, int32_t** host, void** device) {
    MF_REQUIRE(g.inited, MF_E_STATE, "mf_init not called");
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    if (host) *host = g.ranks[rank].h_step;
    if (device) *device = g.ranks[rank].d_step;
    return MF_OK;
}

int mf_decode_status(int rank, int* status, int clear) {
    MF_REQUIRE(status, MF_E_INVALID, "null status");
    MF_REQUIRE(g.inited && rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaStreamSynchronize(r.stream));
    int v = 0;
    MF_CK(cudaMemcpy(&v, (int*)r.d_step + MF_STEP_DSTATUS, sizeof(int), cudaMemcpyDeviceToHost));
    *status = v;
    if (clear) {
        MF_CK(cudaMemset((int*)r.d_step + MF_STEP_DSTATUS, 0, sizeof(int)));
        r.h_step[MF_STEP_DSTATUS] = 0;
    }
    return MF_OK;
}

int mf_timer_start(int rank) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_CK(cudaSetDevice(r.device));
    if (!r.ev_start) {
        MF_CK(cudaEventCreate(&r.ev_start));
        MF_CK(cudaEventCreate(&r.ev_stop));
    }
    MF_CK(cudaEventRecord(r.ev_start, r.stream));
    return MF_OK;
}

int mf_timer_stop(int rank, float* ms) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size() && ms, MF_E_INVALID, "bad arguments");
    Rank& r = g.ranks[rank];
    MF_REQUIRE(r.ev_start, MF_E_STATE, "mf_timer_start not called");
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaEventRecord(r.ev_stop, r.stream));
    MF_CK(cudaEventSynchronize(r.ev_stop));
    MF_CK(cudaEventElapsedTime(ms, r.ev_start, r.ev_stop));
    return MF_OK;
}

int mf_sync(int rank) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    MF_CK(cudaSetDevice(g.ranks[rank].device));
    MF_CK(cudaStreamSynchronize(g.ranks[rank].stream));
    return MF_OK;
}

int mf_begin_frame(int rank, int frame_id) { return mf_begin_frame_ex(rank, frame_id, 0); }

int mf_begin_frame_ex(int rank, int frame_id, int flags) {
    MF_REQUIRE(g.inited, MF_E_STATE, "mf_init not called");
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_REQUIRE(r.recording < 0 && r.pending < 0, MF_E_STATE, "begin_frame while a frame is open");
    MF_CK(cudaSetDevice(r.device));
    r.pending = frame_id;
    if (r.frames.count(frame_id)) return MF_FRAME_REPLAY;
    // Capture: the step record upload is the first node of the graph, so every
    // replay reads the host values current at launch time.
    MF_CK(cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal));
    r.recording = frame_id;
    cudaError_t e = (flags & MF_FRAME_NO_UPLOAD)
                        ? cudaSuccess
                        : cudaMemcpyAsync(r.d_step, r.h_step, MF_STEP_RECORD_BYTES, cudaMemcpyHostToDevice, r.stream);
    if (e != cudaSuccess) {
        cudaGraph_t gr = nullptr;
        cudaStreamEndCapture(r.stream, &gr);
        if (gr) cudaGraphDestroy(gr);
        r.recording = -1;
        r.pending = -1;
        return fail(MF_E_CUDA, "step upload during capture: %s", cudaGetErrorString(e));
    }
    return MF_FRAME_RECORD;
}

static int end_frame_impl(int rank, bool wait) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_REQUIRE(r.pending >= 0, MF_E_STATE, "end_frame without begin_frame");
    MF_CK(cudaSetDevice(r.device));
    const int id = r.pending;
    r.pending = -1;
    if (r.recording >= 0) {
        r.recording = -1;
        cudaGraph_t gr = nullptr;
        MF_CK(cudaStreamEndCapture(r.stream, &gr));
        cudaGraphExec_t ex = nullptr;
        cudaError_t e = cudaGraphInstantiate(&ex, gr, 0);
        cudaGraphDestroy(gr);
        if (e != cudaSuccess) return fail(MF_E_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
        r.frames[id] = ex;
    }
    MF_CK(cudaGraphLaunch(r.frames[id], r.stream));
    if (wait) MF_CK(cudaStreamSynchronize(r.stream));
    return MF_OK;
}

int mf_end_frame(int rank) { return end_frame_impl(rank, true); }

int mf_abort_frame(int rank) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_CK(cudaSetDevice(r.device));
    if (r.recording >= 0) {
        cudaGraph_t gr = nullptr;
        cudaStreamEndCapture(r.stream, &gr);
        if (gr) cudaGraphDestroy(gr);
        cudaGetLastError();
    }
    r.recording = -1;
    r.pending = -1;
    return MF_OK;
}
int mf_end_frame_async(int rank) { return end_frame_impl(rank, false); }

int mf_drop_frames(int rank, int first_id, int last_id) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaStreamSynchronize(r.stream));
    for (auto it = r.frames.begin(); it != r.frames.end();) {
        if (it->first >= first_id && it->first <= last_id) {
            cudaGraphExecDestroy(it->second);
            it = r.frames.erase(it);
        } else {
            ++it;
        }
    }
    return MF_OK;
}

int mf_reset_frames(int rank) {
    MF_REQUIRE(rank >= 0 && rank < (int)g.ranks.size(), MF_E_INVALID, "rank %d out of range", rank);
    Rank& r = g.ranks[rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaStreamSynchronize(r.stream));
    for (auto& kv : r.frames) cudaGraphExecDestroy(kv.second);
    r.frames.clear();
    return MF_OK;
}

// ===================================================================== token-loop ops

int mf_rope_table(float* out, int n_pos, int d_rot, float base) {
    MF_REQUIRE(out && n_pos > 0 && d_rot > 0 && d_rot % 2 == 0, MF_E_INVALID, "bad rope arguments");
    const int half = d_rot / 2;
    std::vector<float> freq(half);
    // src/ops/kernels.cpp:72-73 with the float overloads of pow/cos/sin
    for (int i = 0; i < half; ++i) freq[i] = 1.0f / powf(base, 2.0f * i / d_rot);
    for (int p = 0; p < n_pos; ++p) {
        for (int i = 0; i < half; ++i) {
            const float angle = p * freq[i];
            out[((size_t)p * half + i) * 2 + 0] = cosf(angle);
            out[((size_t)p * half + i) * 2 + 1] = sinf(angle);
        }
    }
    return MF_OK;
}

int mf_embed_step(float* x, const void* emb, int dtype, int vocab, int d_model, const void* step_state,
                  void* stream) {
    MF_REQUIRE(x && emb && step_state, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(d_model > 0 && vocab > 0, MF_E_INVALID, "bad sizes");
    const void* fn = dtype == MF_F32   ? (const void*)&mf::embed_kernel<mf::W_F32>
                     : dtype == MF_F16 ? (const void*)&mf::embed_kernel<mf::W_F16>
                                       : (const void*)&mf::embed_kernel<mf::W_BF16>;
    const mf::StepState* st = (const mf::StepState*)step_state;
    void* args[] = {&x, (void*)&emb, &d_model, &vocab, (void*)&st};
    const int blocks = (d_model + 1023) / 1024;
    MF_CK(launch(fn, dim3(blocks), dim3(256), 0, resolve(stream), args));
    return MF_OK;
}

int mf_rmsnorm_matmul(float* y, const float* x, const float* norm_w, float eps, const void* w, int dtype, int d_out,
                      int d_in, void* stream) {
    MF_REQUIRE(y && x && norm_w && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    mf::GemvParams p = {};
    p.w = w;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = y;
    p.rows = d_out;
    p.K = d_in;
    return run_gemv(dtype, mf::X_NORM, mf::Y_STORE, p, d_out, resolve(stream));
}

int mf_matmul_residual(float* x, const float* a, const void* w, int dtype, int d_out, int d_in, void* stream) {
    MF_REQUIRE(x && a && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    mf::GemvParams p = {};
    p.w = w;
    p.x = a;
    p.y = x;
    p.rows = d_out;
    p.K = d_in;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_RESID, p, d_out, resolve(stream));
}

int mf_swiglu_matmul(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up, int dtype,
                     int d_ff, int d_in, void* stream) {
    MF_REQUIRE(h && x && norm_w && w_gate_up, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    mf::GemvParams p = {};
    p.w = w_gate_up;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = h;
    p.rows = 2 * d_ff;
    p.K = d_in;
    return run_gemv(dtype, mf::X_NORM, mf::Y_SWIGLU, p, d_ff, resolve(stream));
}

size_t mf_attn_workspace_bytes(int n_heads, int n_kv_heads, int d_head, int n_split) {
    if (n_kv_heads <= 0 || n_heads <= 0 || n_split <= 0) return 0;
    return mf::attn_ws_layout(n_kv_heads, n_split, n_heads / n_kv_heads).total;
}

int mf_attn_default_split(int n_kv_heads, int max_seq) {
    if (n_kv_heads <= 0) return 1;
    int sms = num_sms();
    static const int ctas_per_sm = env_int("MF_ATT_CTAS_PER_SM", mf::ATT_CTAS_PER_SM);
    int s = sms * ctas_per_sm / n_kv_heads;
    if (s < 1) s = 1;
    const int max_useful = (max_seq + mf::ATT_MIN_CHUNK - 1) / mf::ATT_MIN_CHUNK;
    if (s > max_useful) s = max_useful;
    if (s > mf::attn_max_split(16)) s = mf::attn_max_split(16);
    return s < 1 ? 1 : s;
}

int mf_attn_decode(const mf_attn_desc* d, void* stream) {
    MF_REQUIRE(d, MF_E_INVALID, "null descriptor");
    MF_REQUIRE(d->qkv && d->q_norm_w && d->k_norm_w && d->rope_table && d->k_cache && d->v_cache && d->step_state &&
                   d->out && d->workspace,
               MF_E_INVALID, "null pointer in attention descriptor");
    MF_REQUIRE(d->d_head == mf::ATT_D, MF_E_UNSUPPORTED, "d_head %d (kernel is built for 128)", d->d_head);
    MF_REQUIRE(d->n_kv_heads > 0 && d->n_heads % d->n_kv_heads == 0, MF_E_INVALID, "n_heads %% n_kv_heads != 0");
    MF_REQUIRE(d->n_split >= 1 && d->max_seq >= 1, MF_E_INVALID, "bad n_split/max_seq");
    const int G = d->n_heads / d->n_kv_heads;
    MF_REQUIRE(d->kv_dtype == MF_F32 || d->kv_dtype == MF_BF16, MF_E_UNSUPPORTED, "KV cache dtype %d (f32 or bf16)",
               d->kv_dtype);
    const void* fn = mf::attn_kernel_ptr(G, d->kv_dtype);
    MF_REQUIRE(fn, MF_E_UNSUPPORTED, "%d query heads per KV head has no kernel", G);
    MF_REQUIRE(d->n_split <= mf::attn_max_split(G), MF_E_UNSUPPORTED, "n_split %d above %d", d->n_split,
               mf::attn_max_split(G));
    const size_t smem = mf::attn_smem_bytes(G);
    int bps = 0;
    int rc = prepare(fn, mf::ATT_WARPS * 32, smem, &bps);
    if (rc) return rc;
    char* ws = (char*)d->workspace;
    const mf::AttnWsLayout L = mf::attn_ws_layout(d->n_kv_heads, d->n_split, G);
    mf::AttnParams p = {};
    p.qkv = d->qkv;
    p.q_norm_w = d->q_norm_w;
    p.k_norm_w = d->k_norm_w;
    p.eps = d->eps;
    p.rope = (const float2*)d->rope_table;
    p.k_cache = d->k_cache;
    p.v_cache = d->v_cache;
    p.max_seq = d->max_seq;
    p.pos_ptr = &((const mf::StepState*)d->step_state)->pos;
    p.out = d->out;
    p.counters = (int*)(ws + L.cnt);
    p.part_ml = (float*)(ws + L.ml);
    p.part_o = (float*)(ws + L.o);
    p.group_ml = (float*)(ws + L.gml);
    p.group_o = (float*)(ws + L.go);
    p.n_heads = d->n_heads;
    p.n_kv_heads = d->n_kv_heads;
    p.n_split = d->n_split;
    void* args[] = {&p};
    MF_CK(launch(fn, dim3(d->n_split, d->n_kv_heads), dim3(mf::ATT_WARPS * 32), smem, resolve(stream), args));
    return MF_OK;
}

int mf_router_topk(int* ids, float* weights, float* scores, const float* x, const float* norm_w, float eps,
                   const float* w_router, int d_model, int n_experts, int k, void* stream) {
    MF_REQUIRE(ids && weights && scores && x && norm_w && w_router, MF_E_INVALID, "null argument");
    MF_REQUIRE(n_experts >= 1 && n_experts <= 256, MF_E_UNSUPPORTED, "n_experts %d (1..256)", n_experts);
    MF_REQUIRE(k >= 1 && k <= n_experts && k <= 32, MF_E_INVALID, "k %d", k);
    MF_REQUIRE(d_model > 0 && d_model % 16 == 0, MF_E_INVALID, "d_model must be a positive multiple of 16");
    cudaStream_t st = resolve(stream);
    mf::GemvParams p = {};
    p.w = w_router;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = scores;
    p.rows = n_experts;
    p.K = d_model;
    int rc = run_gemv(MF_F32, mf::X_NORM, mf::Y_STORE, p, n_experts, st);
    if (rc) return rc;
    void* args[] = {(void*)&scores, &n_experts, &k, &ids, &weights};
    MF_CK(launch((const void*)&mf::topk_softmax_kernel, dim3(1), dim3(32), 0, st, args));
    return MF_OK;
}

int mf_allreduce_router_topk(int* ids, float* weights, float* scores, const float* x_res, float* x_out,
                             const float* norm_w, float eps, const float* w_router, int d_model, int n_experts, int k,
                             mf_comm* c, int seq, const void* step_state, void* stream) {
    MF_REQUIRE(ids && weights && scores, MF_E_INVALID, "null argument");
    MF_REQUIRE(n_experts >= 1 && n_experts <= 256, MF_E_UNSUPPORTED, "n_experts %d (1..256)", n_experts);
    MF_REQUIRE(k >= 1 && k <= n_experts && k <= 32, MF_E_INVALID, "k %d", k);
    int rc = mf_allreduce_rmsnorm_matmul(scores, x_res, x_out, norm_w, eps, w_router, MF_F32, n_experts, d_model, c,
                                         seq, step_state, stream);
    if (rc) return rc;
    void* args[] = {(void*)&scores, &n_experts, &k, &ids, &weights};
    MF_CK(launch((const void*)&mf::topk_softmax_kernel, dim3(1), dim3(32), 0, resolve(stream), args));
    return MF_OK;
}

int mf_moe_swiglu(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up_exps, int dtype,
                  const int* ids, int k, int d_ff, int d_in, void* stream) {
    MF_REQUIRE(h && x && norm_w && w_gate_up_exps && ids, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(k >= 1 && k <= 32 && d_ff > 0, MF_E_INVALID, "bad k/d_ff (k must be 1..32)");
    mf::GemvParams p = {};
    p.w = w_gate_up_exps;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = h;
    p.rows = 2 * d_ff * k;
    p.K = d_in;
    p.expert_ids = ids;
    p.rows_per_expert = 2 * d_ff;
    return run_gemv(dtype, mf::X_NORM, mf::Y_SWIGLU, p, (long long)d_ff * k, resolve(stream));
}

int mf_moe_down_residual(float* x, const float* h, const void* w_down_exps, int dtype, const int* ids,
                         const float* weights, int k, int d_model, int d_ff, void* stream) {
    MF_REQUIRE(x && h && w_down_exps && ids && weights, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(k >= 1 && k <= 8, MF_E_UNSUPPORTED, "k %d (grouped down projection supports 1..8)", k);
    mf::GemvParams p = {};
    p.w = w_down_exps;
    p.x = h;
    p.y = x;
    p.rows = d_model;
    p.K = d_ff;
    p.expert_ids = ids;
    p.expert_w = weights;
    p.rows_per_expert = d_model;
    p.n_slots = k;
    MF_REQUIRE(d_ff > 0 && d_ff % 16 == 0 && d_model > 0, MF_E_INVALID, "bad d_ff/d_model");
    MF_REQUIRE(((uintptr_t)w_down_exps) % 16 == 0 && ((uintptr_t)h) % 16 == 0, MF_E_INVALID,
               "weights and h must be 16-byte aligned");
    const int tr = try_moe_down_tma(dtype, p, resolve(stream), false);
    if (tr < 0) return tr;
    if (tr == 1) return MF_OK;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_MOE_DOWN, p, d_model, resolve(stream));
}

int mf_moe_ffn(float* x, float* h, const float* norm_w, float eps, const float* w_router, const void* w_gate_up_exps,
               const void* w_down_exps, int dtype, float* scores, int* ids, float* weights, int d_model, int d_ff,
               int n_experts, int k, void* stream) {
    MF_REQUIRE(x && h && norm_w && w_router && w_gate_up_exps && w_down_exps && scores && ids && weights, MF_E_INVALID,
               "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(k >= 1 && k <= 8 && d_ff > 0 && d_ff % 16 == 0 && d_model > 0 && d_model % 16 == 0, MF_E_INVALID,
               "bad k/d_ff/d_model (k 1..8, sizes multiples of 16)");
    MF_REQUIRE(((uintptr_t)w_gate_up_exps | (uintptr_t)w_down_exps | (uintptr_t)x | (uintptr_t)h) % 16 == 0,
               MF_E_INVALID, "operands must be 16-byte aligned");
    cudaStream_t st = resolve(stream);
    int rc = mf_router_topk(ids, weights, scores, x, norm_w, eps, w_router, d_model, n_experts, k, st);
    if (rc) return rc;
    mf::GemvParams g = {};
    g.w = w_gate_up_exps;
    g.x = x;
    g.nw = norm_w;
    g.eps = eps;
    g.y = h;
    g.rows = 2 * d_ff * k;
    g.K = d_model;
    g.expert_ids = ids;
    g.rows_per_expert = 2 * d_ff;
    // the down projection may read the ids before its dependency wait only
    // behind the grouped TMA gate/up kernel (which waits for the router
    // before letting it launch)
    const int tg = try_gemv_tma(dtype, mf::X_NORM, mf::Y_SWIGLU, g, st);
    if (tg < 0) return tg;
    if (tg == 0) {
        rc = run_gemv(dtype, mf::X_NORM, mf::Y_SWIGLU, g, (long long)d_ff * k, st);
        if (rc) return rc;
    }
    mf::GemvParams q = {};
    q.w = w_down_exps;
    q.x = h;
    q.y = x;
    q.rows = d_model;
    q.K = d_ff;
    q.expert_ids = ids;
    q.expert_w = weights;
    q.rows_per_expert = d_model;
    q.n_slots = k;
    const int td = try_moe_down_tma(dtype, q, st, tg == 1);
    if (td < 0) return td;
    if (td == 1) return MF_OK;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_MOE_DOWN, q, d_model, st);
}

size_t mf_lm_head_workspace_bytes(void) { return 256 + (size_t)LMH_MAX_GRID * (sizeof(float) + sizeof(int)); }

int mf_lm_head(float* logits, const float* x, const float* norm_w, float eps, const void* w, int dtype, int vocab,
               int d_model, int vocab_offset, void* step_state, void* workspace, void* stream) {
    MF_REQUIRE(logits && x && norm_w && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(!step_state || workspace, MF_E_INVALID, "argmax needs a workspace");
    mf::GemvParams p = {};
    p.w = w;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = logits;
    p.rows = vocab;
    p.K = d_model;
    p.vocab_offset = vocab_offset;
    if (step_state) {
        char* ws = (char*)workspace;
        p.counter = (int*)ws;
        p.best_val = (float*)(ws + 256);
        p.best_idx = (int*)(ws + 256 + (size_t)LMH_MAX_GRID * sizeof(float));
        p.step = (int*)step_state;
    }
    return run_gemv(dtype, mf::X_NORM, mf::Y_STORE, p, vocab, resolve(stream), LMH_MAX_GRID);
}

// ===================================================================== tensor parallelism

int mf_comm_create(int rank, int tp_rank, int tp_size, int max_floats, int gather_floats, mf_comm** out) {
    return mf_comm_create_ex(rank, tp_rank, tp_size, max_floats, gather_floats, 0, out);
}

int mf_comm_create_ex(int rank, int tp_rank, int tp_size, int max_floats, int gather_floats, size_t bulk_floats,
                      mf_comm** out) {
    MF_REQUIRE(out, MF_E_INVALID, "null output");
    MF_REQUIRE(bulk_floats % 4 == 0, MF_E_INVALID, "bulk_floats must be a multiple of 4");
    MF_REQUIRE(g.inited && rank >= 0 && rank < (int)g.ranks.size(), MF_E_STATE, "mf_init first (rank %d)", rank);
    MF_REQUIRE(tp_size >= 1 && tp_size <= MF_TP_MAX && tp_rank >= 0 && tp_rank < tp_size, MF_E_INVALID,
               "tp_rank %d / tp_size %d", tp_rank, tp_size);
    MF_REQUIRE(max_floats > 0 && max_floats % 4 == 0 && gather_floats >= 0, MF_E_INVALID,
               "max_floats must be a positive multiple of 4");
    MF_CK(cudaSetDevice(g.ranks[rank].device));
    auto c = std::make_unique<mf_comm>();
    c->rank = rank;
    c->layout = mf::comm_layout(max_floats, gather_floats, bulk_floats);
    MF_REQUIRE(c->layout.total < (1ull << 32), MF_E_INVALID, "exchange region too large");
    MF_CK(cudaMalloc((void**)&c->region, c->layout.total));
    cudaError_t e = cudaMemset(c->region, 0, c->layout.total);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(c->region);
        return fail(MF_E_CUDA, "exchange region: %s", cudaGetErrorString(e));
    }
    mf::CommDev& d = c->dev;
    d.tp_rank = tp_rank;
    d.tp_size = tp_size;
    d.max_floats = max_floats;
    d.gather_floats = gather_floats;
    // MF_COMM_TIMEOUT_MS: how long an exchange wait polls before giving up
    d.timeout_ns = 1000000ull * (unsigned long long)std::max(1, env_int("MF_COMM_TIMEOUT_MS", 1000));
    d.off_recv = (uint32_t)c->layout.recv;
    d.off_best = (uint32_t)c->layout.best;
    d.off_gather = (uint32_t)c->layout.gather;
    d.off_local = (uint32_t)c->layout.local;
    d.off_flags = (uint32_t)c->layout.flags;
    d.off_bulk = (uint32_t)c->layout.bulk;
    d.bulk_floats = bulk_floats;
    d.base[tp_rank] = c->region;
    c->connected = tp_size == 1;
    *out = c.release();
    return MF_OK;
}

int mf_comm_handle(const mf_comm* c, void* out, size_t n) {
    MF_REQUIRE(c && out && n >= MF_COMM_HANDLE_BYTES, MF_E_INVALID, "bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) <= MF_COMM_HANDLE_BYTES, "IPC handle size");
    MF_CK(cudaSetDevice(g.ranks[c->rank].device));
    cudaIpcMemHandle_t h;
    MF_CK(cudaIpcGetMemHandle(&h, c->region));
    std::memset(out, 0, MF_COMM_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof(h));
    return MF_OK;
}

int mf_comm_connect(mf_comm* c, const void* handles, size_t n) {
    MF_REQUIRE(c && handles, MF_E_INVALID, "null argument");
    const int T = c->dev.tp_size;
    MF_REQUIRE(n == (size_t)T * MF_COMM_HANDLE_BYTES, MF_E_INVALID, "expected %d handles", T);
    MF_REQUIRE(!c->connected || T == 1, MF_E_STATE, "already connected");
    MF_CK(cudaSetDevice(g.ranks[c->rank].device));
    cudaIpcMemHandle_t own;
    MF_CK(cudaIpcGetMemHandle(&own, c->region));
    for (int r = 0; r < T; ++r) {
        if (r == c->dev.tp_rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const char*)handles + (size_t)r * MF_COMM_HANDLE_BYTES, sizeof(h));
        if (std::memcmp(&h, &own, sizeof(h)) == 0) {
            // this rank's own handle in a peer's place: the peer slot maps to
            // this region (a loopback whose peer never sends; exercises the
            // waits' time limit)
            c->dev.base[r] = c->region;
            continue;
        }
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void* q : c->opened) cudaIpcCloseMemHandle(q);
            c->opened.clear();
            return fail(MF_E_CUDA, "open peer %d exchange region: %s", r, cudaGetErrorString(e));
        }
        c->opened.push_back(p);
        c->dev.base[r] = (char*)p;
    }
    c->connected = true;
    return MF_OK;
}

int mf_comm_status(mf_comm* c, int* status, int clear) {
    MF_REQUIRE(c && status, MF_E_INVALID, "null argument");
    Rank& r = g.ranks[c->rank];
    MF_CK(cudaSetDevice(r.device));
    MF_CK(cudaStreamSynchronize(r.stream));
    int* dst = (int*)(c->region + c->layout.local + offsetof(mf::CommLocal, status));
    MF_CK(cudaMemcpy(status, dst, sizeof(int), cudaMemcpyDeviceToHost));
    if (clear) MF_CK(cudaMemset(dst, 0, sizeof(int)));
    return MF_OK;
}

size_t mf_topk_workspace_bytes(int n, int k) {
    if (n <= 0 || k <= 0) return 0;
    const size_t grid = ((size_t)n + mf::TOPK_CHUNK - 1) / mf::TOPK_CHUNK;
    return 256 + grid * (size_t)k * (sizeof(float) + sizeof(int));
}

int mf_topk(const float* x, int n, int k, int* ids, float* vals, void* workspace, size_t workspace_bytes,
            void* stream) {
    MF_REQUIRE(x && ids && vals && workspace, MF_E_INVALID, "null argument");
    MF_REQUIRE(k >= 1 && k <= mf::TOPK_MAX && n >= k, MF_E_INVALID, "need 1 <= k <= %d and k <= n", mf::TOPK_MAX);
    MF_REQUIRE(workspace_bytes >= mf_topk_workspace_bytes(n, k), MF_E_INVALID, "top-k workspace too small");
    MF_REQUIRE(((uintptr_t)workspace & 15) == 0, MF_E_INVALID, "workspace must be 16-byte aligned");
    const int grid = (n + mf::TOPK_CHUNK - 1) / mf::TOPK_CHUNK;
    const size_t smem = 2 * (size_t)std::max(mf::TOPK_CHUNK, grid * k) * sizeof(float);
    MF_REQUIRE(smem <= 200 * 1024, MF_E_UNSUPPORTED, "n * k too large for one merge CTA");
    // the shared-memory opt-in only ever grows (per device), so a concurrent
    // call with a smaller request cannot lower it under this launch
    int bps = 0;
    int rc = prepare((const void*)&mf::topk_kernel, mf::TOPK_THREADS, smem, &bps);
    if (rc) return rc;
    unsigned int* counter = (unsigned int*)workspace;
    float* cand_v = (float*)((char*)workspace + 256);
    int* cand_i = (int*)(cand_v + (size_t)grid * k);
    void* args[] = {(void*)&x, (void*)&n, (void*)&k, (void*)&ids, (void*)&vals, (void*)&cand_v, (void*)&cand_i,
                    (void*)&counter};
    MF_CK(launch((const void*)&mf::topk_kernel, dim3(grid), dim3(mf::TOPK_THREADS), smem,
                 mf::resolve_stream(stream), args));
    return MF_OK;
}

int mf_sample_step(const int* cand_ids, const float* cand_vals, int top_k, float temp, float top_p, float min_p,
                   const float* draws, int n_draws, void* step_state, int* out_ids, int* flags, void* stream) {
    MF_REQUIRE(cand_ids && cand_vals && draws && step_state && out_ids && flags, MF_E_INVALID, "null argument");
    MF_REQUIRE(top_k >= 1 && top_k + 1 <= mf::TOPK_MAX && top_k <= mf::SAMPLE_MAX_K, MF_E_INVALID,
               "top_k must leave room for top_k + 1 candidates");
    MF_REQUIRE(temp > 0.f && top_p >= 0.f && top_p <= 1.f && min_p >= 0.f && min_p <= 1.f && n_draws > 0,
               MF_E_INVALID, "bad sampling parameters");
    mf::StepState* st = (mf::StepState*)step_state;
    void* args[] = {(void*)&cand_ids, (void*)&cand_vals, &top_k, &temp, &top_p, &min_p, (void*)&draws, &n_draws,
                    &st, &out_ids, &flags};
    MF_CK(launch((const void*)&mf::sample_step_kernel, dim3(1), dim3(32), 0, resolve(stream), args));
    return MF_OK;
}

int mf_comm_bulk_ptr(const mf_comm* c, int slot, float** out) {
    MF_REQUIRE(c && out && (slot == 0 || slot == 1), MF_E_INVALID, "bad arguments");
    MF_REQUIRE(c->dev.bulk_floats > 0, MF_E_STATE, "exchange region has no bulk slots");
    *out = (float*)(c->region + c->layout.bulk) + (size_t)slot * c->dev.bulk_floats;
    return MF_OK;
}

int mf_bulk_allreduce(float* x, size_t n, mf_comm* c, int slot, unsigned long long epoch, void* stream) {
    MF_REQUIRE(x && c && (slot == 0 || slot == 1) && epoch > 0, MF_E_INVALID, "bad arguments");
    MF_REQUIRE(c->connected, MF_E_STATE, "mf_comm_connect first");
    MF_REQUIRE(n > 0 && n % 4 == 0 && n <= c->dev.bulk_floats, MF_E_INVALID,
               "n must be a positive multiple of 4 within the bulk slot (%zu floats)", c->dev.bulk_floats);
    MF_REQUIRE(((uintptr_t)x & 15) == 0, MF_E_INVALID, "x must be 16-byte aligned");
    const size_t n4 = n / 4;
    long long grid = (long long)((n4 + 255) / 256);
    grid = std::min<long long>(grid, (long long)num_sms() * 4);
    const mf::CommDev dev = c->dev;
    cudaStream_t st = mf::resolve_stream(stream);
    // flags rise by two per exchange: partial complete, then reduced slice complete
    unsigned long long f1 = 2 * epoch - 1, f2 = 2 * epoch;
    {
        const long long g1 = std::max<long long>(1, std::min<long long>(grid / dev.tp_size + 1, grid));
        void* args[] = {(void*)&n4, (void*)&dev, (void*)&slot, (void*)&f1};
        MF_CK(launch((const void*)&mf::bulk_reduce_kernel, dim3((unsigned)g1), dim3(256), 0, st, args));
    }
    void* args[] = {(void*)&x, (void*)&n4, (void*)&dev, (void*)&slot, (void*)&f2};
    MF_CK(launch((const void*)&mf::bulk_gather_kernel, dim3((unsigned)grid), dim3(256), 0, st, args));
    return MF_OK;
}

int mf_comm_gather_ptr(const mf_comm* c, float** logits) {
    MF_REQUIRE(c && logits && c->dev.gather_floats > 0, MF_E_INVALID, "no gather buffer");
    *logits = (float*)(c->region + c->layout.gather);
    return MF_OK;
}

void mf_comm_destroy(mf_comm* c) {
    if (!c) return;
    if (c->rank < (int)g.ranks.size()) {
        cudaSetDevice(g.ranks[c->rank].device);
        cudaDeviceSynchronize();
    }
    for (void* q : c->opened) cudaIpcCloseMemHandle(q);
    cudaFree(c->region);
    delete c;
}

namespace {
int comm_ready(const mf_comm* c, int seq, const void* step_state) {
    MF_REQUIRE(c && c->connected, MF_E_STATE, "exchange not connected (mf_comm_connect)");
    MF_REQUIRE(seq >= 0 && seq < mf::COMM_SEQ_GREEDY, MF_E_INVALID, "exchange number %d outside [0, %d)", seq,
               mf::COMM_SEQ_GREEDY);
    MF_REQUIRE(step_state, MF_E_INVALID, "the exchange needs the step record (frame tag)");
    return MF_OK;
}
}  // namespace

int mf_matmul_push(const float* a, const void* w, int dtype, int d_out, int d_in, mf_comm* c, int seq,
                   const void* step_state, void* stream) {
    MF_REQUIRE(a && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(d_out <= c->dev.max_floats, MF_E_INVALID, "d_out %d exceeds the exchange slot (%d)", d_out,
               c->dev.max_floats);
    mf::GemvParams p = {};
    p.w = w;
    p.x = a;
    p.rows = d_out;
    p.K = d_in;
    p.comm = c->dev;
    p.ar_seq = seq;
    p.step = (int*)step_state;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_PUSH, p, d_out, resolve(stream));
}

int mf_allreduce_rmsnorm_matmul(float* y, const float* x_res, float* x_out, const float* norm_w, float eps,
                                const void* w, int dtype, int d_out, int d_in, mf_comm* c, int seq,
                                const void* step_state, void* stream) {
    MF_REQUIRE(y && x_res && x_out && norm_w && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(x_out != x_res, MF_E_INVALID, "x_out must differ from x_res (other CTAs still read it)");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(d_in <= c->dev.max_floats, MF_E_INVALID, "d_in %d exceeds the exchange slot", d_in);
    mf::GemvParams p = {};
    p.w = w;
    p.x_res = x_res;
    p.x_out = x_out;
    p.nw = norm_w;
    p.eps = eps;
    p.y = y;
    p.rows = d_out;
    p.K = d_in;
    p.comm = c->dev;
    p.ar_seq = seq;
    p.step = (int*)step_state;
    return run_gemv(dtype, mf::X_AR_NORM, mf::Y_STORE, p, d_out, resolve(stream));
}

int mf_allreduce_swiglu_matmul(float* h, const float* x_res, float* x_out, const float* norm_w, float eps,
                               const void* w_gate_up, int dtype, int d_ff, int d_in, mf_comm* c, int seq,
                               const void* step_state, void* stream) {
    MF_REQUIRE(h && x_res && x_out && norm_w && w_gate_up, MF_E_INVALID, "null argument");
    MF_REQUIRE(x_out != x_res, MF_E_INVALID, "x_out must differ from x_res (other CTAs still read it)");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(d_in <= c->dev.max_floats, MF_E_INVALID, "d_in %d exceeds the exchange slot", d_in);
    mf::GemvParams p = {};
    p.w = w_gate_up;
    p.x_res = x_res;
    p.x_out = x_out;
    p.nw = norm_w;
    p.eps = eps;
    p.y = h;
    p.rows = 2 * d_ff;
    p.K = d_in;
    p.comm = c->dev;
    p.ar_seq = seq;
    p.step = (int*)step_state;
    return run_gemv(dtype, mf::X_AR_NORM, mf::Y_SWIGLU, p, d_ff, resolve(stream));
}

int mf_allreduce_lm_head(float* logits, const float* x_res, float* x_out, const float* norm_w, float eps,
                         const void* w, int dtype, int vocab, int d_model, int vocab_offset, void* step_state,
                         void* workspace, int gather_logits, mf_comm* c, int seq, void* stream) {
    MF_REQUIRE(logits && x_res && x_out && norm_w && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(x_out != x_res, MF_E_INVALID, "x_out must differ from x_res (other CTAs still read it)");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(!step_state || workspace, MF_E_INVALID, "argmax needs a workspace");
    MF_REQUIRE(step_state && workspace, MF_E_INVALID, "the exchange needs the step record and the workspace");
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(d_model <= c->dev.max_floats, MF_E_INVALID, "d_model %d exceeds the exchange slot", d_model);
    MF_REQUIRE(!gather_logits || (long long)vocab_offset + vocab <= c->dev.gather_floats, MF_E_INVALID,
               "logits rows [%d, %d) outside the gather buffer (%d)", vocab_offset, vocab_offset + vocab,
               c->dev.gather_floats);
    mf::GemvParams p = {};
    p.w = w;
    p.x_res = x_res;
    p.x_out = x_out;
    p.nw = norm_w;
    p.eps = eps;
    p.y = logits;
    p.rows = vocab;
    p.K = d_model;
    p.vocab_offset = vocab_offset;
    p.comm = c->dev;
    p.ar_seq = seq;
    p.gather_logits = gather_logits ? 1 : 0;
    {
        char* ws = (char*)workspace;
        p.counter = (int*)ws;
        p.best_val = (float*)(ws + 256);
        p.best_idx = (int*)(ws + 256 + (size_t)LMH_MAX_GRID * sizeof(float));
        p.step = (int*)step_state;
    }
    return run_gemv(dtype, mf::X_AR_NORM, mf::Y_STORE, p, vocab, resolve(stream), LMH_MAX_GRID);
}

int mf_moe_swiglu_ep(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up_local, int dtype,
                     const int* ids, int k, int d_ff, int d_in, int expert_lo, int n_local, void* stream) {
    MF_REQUIRE(h && x && norm_w && w_gate_up_local && ids, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(k >= 1 && k <= 32 && d_ff > 0 && expert_lo >= 0 && n_local >= 1, MF_E_INVALID,
               "bad k/d_ff/expert range (k must be 1..32)");
    mf::GemvParams p = {};
    p.w = w_gate_up_local;
    p.x = x;
    p.nw = norm_w;
    p.eps = eps;
    p.y = h;
    p.rows = 2 * d_ff * k;
    p.K = d_in;
    p.expert_ids = ids;
    p.rows_per_expert = 2 * d_ff;
    p.ep_lo = expert_lo;
    p.ep_n = n_local;
    return run_gemv(dtype, mf::X_NORM, mf::Y_SWIGLU, p, (long long)d_ff * k, resolve(stream));
}

int mf_moe_down_push(const float* h, const void* w_down_local, int dtype, const int* ids, const float* weights, int k,
                     int d_model, int d_ff, int expert_lo, int n_local, mf_comm* c, int seq, const void* step_state,
                     void* stream) {
    MF_REQUIRE(h && w_down_local && ids && weights, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    MF_REQUIRE(k >= 1 && k <= 8, MF_E_UNSUPPORTED, "k %d (grouped down projection supports 1..8)", k);
    MF_REQUIRE(expert_lo >= 0 && n_local >= 1, MF_E_INVALID, "bad expert range");
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(d_model <= c->dev.max_floats, MF_E_INVALID, "d_model %d exceeds the exchange slot", d_model);
    mf::GemvParams p = {};
    p.w = w_down_local;
    p.x = h;
    p.rows = d_model;
    p.K = d_ff;
    p.expert_ids = ids;
    p.expert_w = weights;
    p.rows_per_expert = d_model;
    p.n_slots = k;
    p.ep_lo = expert_lo;
    p.ep_n = n_local;
    p.comm = c->dev;
    p.ar_seq = seq;
    p.step = (int*)step_state;
    MF_REQUIRE(d_ff % 16 == 0 && ((uintptr_t)w_down_local | (uintptr_t)h) % 16 == 0, MF_E_INVALID,
               "d_ff must be a multiple of 16, weights and h 16-byte aligned");
    const int tr = try_moe_down_tma(dtype, p, resolve(stream), false, true);
    if (tr < 0) return tr;
    if (tr == 1) return MF_OK;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_MOE_PUSH, p, d_model, resolve(stream));
}

int mf_allreduce(float* x_out, const float* x_res, const float* partial, int n, mf_comm* c, int seq,
                 const void* step_state, void* stream) {
    MF_REQUIRE(x_out && x_res && partial && n > 0, MF_E_INVALID, "bad arguments");
    int rc = comm_ready(c, seq, step_state);
    if (rc) return rc;
    MF_REQUIRE(n <= c->dev.max_floats, MF_E_INVALID, "n %d exceeds the exchange slot", n);
    const void* fn = (const void*)&mf::allreduce_kernel;
    mf::CommDev dev = c->dev;
    const mf::StepState* st = (const mf::StepState*)step_state;
    void* args[] = {(void*)&partial, (void*)&x_res, (void*)&x_out, (void*)&n, (void*)&dev, (void*)&seq, (void*)&st};
    MF_CK(launch(fn, dim3(1), dim3(1024), 0, resolve(stream), args));
    return MF_OK;
}

// ===================================================================== single ops

int mf_matmul(float* y, const float* x, const void* w, int dtype, size_t offset, int d_out, int d_in, void* stream) {
    MF_REQUIRE(y && x && w, MF_E_INVALID, "null argument");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    mf::GemvParams p = {};
    p.w = w;
    p.w_offset = offset;
    p.x = x;
    p.y = y;
    p.rows = d_out;
    p.K = d_in;
    return run_gemv(dtype, mf::X_PLAIN, mf::Y_STORE, p, d_out, resolve(stream));
}

int mf_rmsnorm(float* out, const float* x, const float* w, int dim, float eps, int n_rows, void* stream) {
    MF_REQUIRE(out && x && w && dim > 0 && n_rows > 0, MF_E_INVALID, "bad arguments");
    mf::rmsnorm_rows_kernel<<<n_rows, 256, 0, resolve(stream)>>>(out, x, w, dim, eps);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

int mf_softmax(float* out, const float* x, int n, int n_rows, void* stream) {
    MF_REQUIRE(out && x && n > 0 && n_rows > 0, MF_E_INVALID, "bad arguments");
    mf::softmax_rows_kernel<<<n_rows, 256, 0, resolve(stream)>>>(out, x, n);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

int mf_silu(float* out, const float* x, int n, void* stream) {
    MF_REQUIRE(out && x && n > 0, MF_E_INVALID, "bad arguments");
    mf::silu_kernel<<<(n + 255) / 256, 256, 0, resolve(stream)>>>(out, x, n);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

static int rope_impl(float* out, const float* x, int head, int d_head, int d_rot, float base, int pos, int neox,
                     void* stream) {
    MF_REQUIRE(out && x && head >= 0 && d_head > 0 && d_rot > 0 && d_rot <= d_head, MF_E_INVALID, "bad arguments");
    mf::rope_head_kernel<<<1, 128, 0, resolve(stream)>>>(out, x, head, d_head, d_rot, base, pos, neox);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

int mf_neox_rope(float* out, const float* x, int head, int d_head, int d_rot, float base, int pos, void* stream) {
    return rope_impl(out, x, head, d_head, d_rot, base, pos, 1, stream);
}

int mf_il_rope(float* out, const float* x, int head, int d_head, int d_rot, float base, int pos, void* stream) {
    return rope_impl(out, x, head, d_head, d_rot, base, pos, 0, stream);
}

int mf_attn(float* scores, float* out, const float* q, const float* k, const float* v, int seq_len, int d_head,
            int kv_dim, void* stream) {
    MF_REQUIRE(scores && out && q && k && v && seq_len > 0 && d_head > 0 && kv_dim >= d_head, MF_E_INVALID,
               "bad arguments");
    mf::attn_head_kernel<<<1, 256, 0, resolve(stream)>>>(scores, out, q, k, v, seq_len, d_head, kv_dim);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

int mf_route(const float* x, int* ids, float* weights, float* scores, const float* w_router, int d_model,
             int n_experts, int k, void* stream) {
    MF_REQUIRE(x && ids && weights && scores && w_router, MF_E_INVALID, "null argument");
    MF_REQUIRE(n_experts >= 1 && n_experts <= 256, MF_E_UNSUPPORTED, "n_experts %d (1..256)", n_experts);
    MF_REQUIRE(k >= 1 && k <= n_experts && k <= 32, MF_E_INVALID, "k %d", k);
    cudaStream_t st = resolve(stream);
    int rc = mf_matmul(scores, x, w_router, MF_F32, 0, n_experts, d_model, st);
    if (rc) return rc;
    void* args[] = {(void*)&scores, &n_experts, &k, &ids, &weights};
    MF_CK(launch((const void*)&mf::topk_softmax_kernel, dim3(1), dim3(32), 0, st, args));
    return MF_OK;
}

int mf_embed(float* x, const void* w, int dtype, uint32_t token, int d_model, void* stream) {
    MF_REQUIRE(x && w && d_model > 0, MF_E_INVALID, "bad arguments");
    MF_REQUIRE(valid_dtype(dtype), MF_E_INVALID, "bad dtype %d", dtype);
    cudaStream_t st = resolve(stream);
    const int blocks = (d_model + 255) / 256;
    if (dtype == MF_F32) mf::embed_row_kernel<mf::W_F32><<<blocks, 256, 0, st>>>(x, w, token, d_model);
    else if (dtype == MF_F16) mf::embed_row_kernel<mf::W_F16><<<blocks, 256, 0, st>>>(x, w, token, d_model);
    else mf::embed_row_kernel<mf::W_BF16><<<blocks, 256, 0, st>>>(x, w, token, d_model);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

int mf_argmax(const float* logits, int n, int* out, void* stream) {
    MF_REQUIRE(logits && out && n > 0, MF_E_INVALID, "bad arguments");
    mf::argmax_kernel<<<1, 1024, 0, resolve(stream)>>>(logits, n, out);
    MF_CK(cudaGetLastError());
    return MF_OK;
}

}  // extern "C"
