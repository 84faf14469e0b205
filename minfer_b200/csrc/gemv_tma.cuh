// Dense decode GEMV fed by 1-D TMA bulk copies: y = W x (optionally x
// RMS-normalised first) with a store, residual-add or SwiGLU epilogue.
//
// Arithmetic follows the reference's matmul_{fp32,fp16,bf16}
// (src/ops/kernels.cpp:211-343): weights widened exactly to fp32, fp32 FMAs,
// one fp32 result per row (summation order differs: fp32 rounding level).
//
// Why TMA here: at batch 1 a GEMV is one pass over the weights, and the
// register-fed kernel (gemv.cuh) keeps at most 8 x 16 bytes per thread in
// flight, so each CTA walks its rows in latency-bound steps. Here one
// producer lane streams the CTA's contiguous rows into a shared-memory ring
// with cp.async.bulk (whole rows per copy, completion counted in bytes on a
// "full" mbarrier per stage); the bytes in flight per SM are the ring size,
// independent of registers.
//
// CTA layout: warps 0..NWC-1 consume, warp NWC produces. A CTA owns a
// contiguous balanced range of units (rows, or gate/up row pairs). Consumer
// warp w owns a fixed slice of the K columns for every row: its lanes hold
// that slice of x (normalised, for X_NORM) in registers, read the weight
// vectors of each staged row from shared memory, and reduce each row over
// the warp; the per-warp partial of every row goes to shared memory and the
// epilogue sums the NWC partials in a fixed order. A consumer warp arrives on
// the stage's "empty" mbarrier when done with it; the producer refills the
// stage once all NWC warps arrived.
//
// Two CTAs per SM with a 64 KB ring each (measured best in the 8B decode
// step: 283 vs 277 tokens/s for the register-fed kernel alone); rows wider
// than 10 KB (the K = 8192 / 12288 / 25600 projections) stay on the
// register-fed kernel, which measured faster there. Every mbarrier wait is bounded by a
// wall-clock deadline; on expiry the kernel records a status bit, stops
// issuing copies, waits (bounded) for the copies it has in flight and returns.
#pragma once

#include "comm.cuh"
#include "mbarrier.cuh"
#include "mf_common.cuh"

namespace mf {

constexpr int GT_MAX_STAGES = 8;
constexpr uint32_t GT_RING_BYTES = 64 * 1024;
constexpr uint32_t GT_STAGE_TARGET = 32 * 1024;
constexpr int GT_STATUS_TIMEOUT = 1;       // bit set in *status when a wait gave up
constexpr int GT_RG = 4;                   // rows a consumer warp works on together

struct GemvTmaParams {
    const char* w;            // weight rows (dtype of the template), first row 16-byte aligned
    unsigned long long row_bytes;
    int rows;                 // rows of W (Y_SWIGLU: 2 x outputs, gate/up interleaved)
    int K;
    const float* x;
    const float* nw;          // RMSNorm weight (X_NORM)
    float eps;
    float* y;
    int rows_per_stage;       // a multiple of the unit size
    int stages;
    uint32_t stage_bytes;     // rows_per_stage * row_bytes (16-byte multiple)
    int* status;              // timeout bit
    unsigned long long timeout_ns;
    // split-K: a cluster of `ksplit` CTAs shares a row range, CTA rank r of the
    // cluster takes columns [r*K, (r+1)*K) of rows `row_stride` bytes apart
    // (K here is the slice width); rank 0 sums the ranks' partials through
    // distributed shared memory. 1: no split (row_stride == row_bytes).
    int ksplit;
    unsigned long long row_stride;
    // tensor parallelism (X_AR_NORM receive in the prologue, Y_PUSH send in
    // the epilogue; the same exchange protocol as the register-fed kernel)
    CommDev comm;
    int ar_seq;
    const int* step;        // device step record (frame number for the tags)
    const float* x_res;     // X_AR_NORM: residual before the all-reduce (x is then x_out)
    float* x_out;           // X_AR_NORM: residual after it
    // grouped experts (Y_SWIGLU over the k selected experts): logical row r is
    // row r % rows_per_expert of expert expert_ids[r / rows_per_expert], whose
    // matrix starts expert_bytes * id into w. The ids come from the router
    // kernel, so the producer copies only after the dependency wait.
    const int* expert_ids;  // [rows / rows_per_expert] device, or null (dense)
    int rows_per_expert;
    unsigned long long expert_bytes;
    // expert parallelism: only experts [ep_lo, ep_lo + ep_n) are stored here
    // (expert e at local index e - ep_lo); rows of slots routed elsewhere are
    // not copied and their outputs are left unused. ep_n == 0: all local.
    int ep_lo, ep_n;
};

// Y_PUSH: row `row` of this rank's partial, as a tagged word into every
// rank's receive slot of exchange ar_seq.
MF_DEVICE void push_row(const GemvTmaParams& p, int row, float v) {
    const unsigned long long w = tagged(v, comm_tag(__ldcg(p.step + MF_STEP_FRAME), p.ar_seq));
    for (int r = 0; r < p.comm.tp_size; ++r) st_tagged(p.comm.recv(r, p.ar_seq & 1, p.comm.tp_rank) + row, w);
}

// Dynamic shared memory: the ring, then the per-row partial sums [rows of this CTA][NWC].
// J: 16-byte vectors per lane of a row (the warp's K slice is at most 32*J vectors).
template <typename W, int NWC, int J, int XM, int YM>
__global__ void __launch_bounds__((NWC + 1) * 32, 1) gemv_tma_kernel(const GemvTmaParams p) {
    constexpr int VEC = W::VEC;
    constexpr int RU = (YM == Y_SWIGLU) ? 2 : 1;
    extern __shared__ __align__(128) unsigned char gt_smem[];
    __shared__ __align__(8) uint64_t full[GT_MAX_STAGES], empty[GT_MAX_STAGES];
    __shared__ float ss_part[NWC];
    __shared__ int abort_s;
    __shared__ int eid_s[32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long units = p.rows / RU;
    const int ks = p.ksplit;
    const uint32_t krank = ks > 1 ? cluster_rank() : 0u;
    const int blk = blockIdx.x / ks, nblk = gridDim.x / ks;
    const int r0 = (int)((long long)blk * units / nblk) * RU;
    const int r1 = (int)((long long)(blk + 1) * units / nblk) * RU;
    // this CTA's column slice starts kofs bytes into each row
    const unsigned long long kofs = (unsigned long long)krank * p.row_bytes;
    const int nrows = r1 - r0;
    const int nchunks = (nrows + p.rows_per_stage - 1) / p.rows_per_stage;
    const int S = p.stages;
    float* part = reinterpret_cast<float*>(gt_smem + (size_t)S * p.stage_bytes);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NWC);
        }
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned long long deadline = globaltimer_ns() + p.timeout_ns;

    if (warp == NWC) {
        // ---- producer: weights do not depend on earlier kernels, so the ring
        // fills before the dependency wait. The next kernel may launch at once
        // (its CTAs fit beside this one and fill their own rings meanwhile).
        const bool grouped = p.expert_ids != nullptr;
        // grouped: the expert ids are the router's output, so this kernel lets
        // its dependents launch only after its own dependency wait (every
        // thread waits first): a kernel launched after it may then read the
        // ids before its own wait
        if (grouped) pdl_wait();
        pdl_launch_dependents();
        if (lane == 0) {
            if (grouped) {
                const int n_ids = p.rows / p.rows_per_expert;
                for (int i = 0; i < n_ids && i < 32; ++i) eid_s[i] = __ldcg(p.expert_ids + i);
            }
            bool failed = false;
            int c = 0;
            for (; c < nchunks; ++c) {
                const int s = c % S;
                if (c >= S && !mbar_wait(&empty[s], (uint32_t)((c / S - 1) & 1), deadline, failed)) break;
                if (*(volatile int*)&abort_s) break;
                const int rr = min(p.rows_per_stage, nrows - c * p.rows_per_stage);
                const char* src = p.w + (size_t)(r0 + c * p.rows_per_stage) * p.row_stride + kofs;
                if (grouped) {
                    // one copy per run of rows inside one expert stored here (the
                    // bytes announced first: runs of other ranks' experts are skipped)
                    uint32_t bytes = 0;
                    for (int pass = 0; pass < 2; ++pass) {
                        if (pass == 1) mbar_expect_tx(&full[s], bytes);
                        int r = 0;
                        while (r < rr) {
                            const int lr = r0 + c * p.rows_per_stage + r;
                            const int slot = lr / p.rows_per_expert, er = lr - slot * p.rows_per_expert;
                            const int n = min(rr - r, p.rows_per_expert - er);
                            const int e = eid_s[slot] - (p.ep_n ? p.ep_lo : 0);
                            if (p.ep_n == 0 || (e >= 0 && e < p.ep_n)) {
                                if (pass == 0) bytes += (uint32_t)(n * p.row_bytes);
                                else
                                    bulk_load(gt_smem + (size_t)s * p.stage_bytes + (size_t)r * p.row_bytes,
                                              p.w + (size_t)e * p.expert_bytes + (size_t)er * p.row_bytes,
                                              (uint32_t)(n * p.row_bytes), &full[s]);
                            }
                            r += n;
                        }
                    }
                } else if (ks == 1) {
                    const uint32_t bytes = (uint32_t)(rr * p.row_bytes);
                    mbar_expect_tx(&full[s], bytes);
                    bulk_load(gt_smem + (size_t)s * p.stage_bytes, src, bytes, &full[s]);
                } else {  // the slices of consecutive rows are row_stride apart: one copy per row
                    mbar_expect_tx(&full[s], (uint32_t)(rr * p.row_bytes));
                    for (int r = 0; r < rr; ++r)
                        bulk_load(gt_smem + (size_t)s * p.stage_bytes + (size_t)r * p.row_bytes,
                                  src + (size_t)r * p.row_stride, (uint32_t)p.row_bytes, &full[s]);
                }
            }
            if (failed) {
                atomicOr(p.status, GT_STATUS_TIMEOUT);
                abort_s = 1;
            }
            // the CTA may only exit once every copy it issued has landed: wait
            // (bounded) for the stages not yet known complete
            bool drain_failed = false;
            for (int d = max(0, c - S); d < c; ++d)
                mbar_wait(&full[d % S], (uint32_t)((d / S) & 1), deadline + p.timeout_ns, drain_failed);
        }
        if (ks > 1) {
            // the cluster barriers of the split-K epilogue count every thread
            __syncwarp();
            cluster_sync_all();
            cluster_sync_all();
        }
        return;
    }

    // ---- consumers: this warp's K slice [v0, v1) in 16-byte vectors
    const int NV = p.K / VEC;
    const int v0 = warp * NV / NWC, v1 = (warp + 1) * NV / NWC;
    float xr[J][VEC];
    if (p.expert_ids) {
        pdl_wait();
        pdl_launch_dependents();
    } else {
        pdl_launch_dependents();
        pdl_wait();
    }
    if (XM == X_AR_NORM) {
        // all-reduce receive: each CTA sums its slice of x = residual +
        // partial_0 + ... (rank order) into x_out as the tagged words arrive;
        // after a grid barrier (every CTA of the grid is resident: the grid
        // fits the GPU and the next kernel launches only once all of these
        // CTAs started) every consumer reads its K slice of the reduced x
        const uint32_t tag = comm_tag(__ldcg(p.step + MF_STEP_FRAME), p.ar_seq);
        const int slot = p.ar_seq & 1;
        int* cst = &p.comm.local()->status;
        const unsigned long long dl = globaltimer_ns() + p.comm.timeout_ns;
        bool late = false;
        const int e0 = (int)((long long)blockIdx.x * p.K / gridDim.x);
        const int e1 = (int)((long long)(blockIdx.x + 1) * p.K / gridDim.x);
        recv_sum(p.comm, slot, tag, p.x_res, e0 + tid, NWC * 32, e1, dl, &late, cst,
                 [&](int i, float v) { p.x_out[i] = v; });
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
        if (tid == 0) grid_arrive_wait(&p.comm.local()->bar[slot], tag, gridDim.x, dl, &late, cst, COMM_STATUS_AR_TIMEOUT);
        asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int v = v0 + lane + 32 * j;
#pragma unroll
        for (int e = 0; e < VEC; e += 4) {
            float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
            if (v < v1) t = __ldcg(reinterpret_cast<const float4*>(p.x + (size_t)krank * p.K + (size_t)v * VEC + e));
            xr[j][e] = t.x; xr[j][e + 1] = t.y; xr[j][e + 2] = t.z; xr[j][e + 3] = t.w;
            if (XM == X_NORM || XM == X_AR_NORM) {
                ss = fmaf(t.x, t.x, ss);
                ss = fmaf(t.y, t.y, ss);
                ss = fmaf(t.z, t.z, ss);
                ss = fmaf(t.w, t.w, ss);
            }
        }
    }
    if (XM == X_NORM || XM == X_AR_NORM) {
        // src/ops/kernels.cpp:355-363: inv = 1/sqrtf(sum(x^2)/dim + eps); out = inv * x * w
        ss = warp_sum(ss);
        if (lane == 0) ss_part[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
        float tot = 0.f;
        for (int i = 0; i < NWC; ++i) tot += ss_part[i];
        const float inv = 1.0f / sqrtf(tot / (float)p.K + p.eps);
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int v = v0 + lane + 32 * j;
            if (v < v1) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) xr[j][e] = (inv * xr[j][e]) * __ldg(p.nw + (size_t)v * VEC + e);
            }
        }
    }

    bool failed = false;
    for (int c = 0; c < nchunks; ++c) {
        const int s = c % S;
        if (!mbar_wait(&full[s], (uint32_t)((c / S) & 1), deadline, failed)) break;
        const unsigned char* st = gt_smem + (size_t)s * p.stage_bytes;
        const int rr = min(p.rows_per_stage, nrows - c * p.rows_per_stage);
        // rows in groups of GT_RG: all their vectors are loaded before any is
        // used and their warp reductions run interleaved, so the shared-memory
        // and shuffle latencies of one row overlap the others'
        int rg = 0;
        for (; rg + GT_RG <= rr; rg += GT_RG) {
            uint4 wv[GT_RG][J];
#pragma unroll
            for (int r = 0; r < GT_RG; ++r) {
                const unsigned char* row = st + (size_t)(rg + r) * p.row_bytes;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int v = v0 + lane + 32 * j;
                    wv[r][j] = v < v1 ? *reinterpret_cast<const uint4*>(row + (size_t)v * 16) : make_uint4(0u, 0u, 0u, 0u);
                }
            }
            float acc[GT_RG];
#pragma unroll
            for (int r = 0; r < GT_RG; ++r) {
                acc[r] = 0.f;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    float wf[VEC];
                    unpack16<W>(wv[r][j], wf);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[r] = fmaf(xr[j][e], wf[e], acc[r]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int r = 0; r < GT_RG; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            if (lane < GT_RG) {
                float a = acc[0];
#pragma unroll
                for (int r = 1; r < GT_RG; ++r)
                    if (lane == r) a = acc[r];
                part[(size_t)(c * p.rows_per_stage + rg + lane) * NWC + warp] = a;
            }
        }
        // the rest one row at a time (wide rows: a stage holds fewer than GT_RG)
        for (; rg < rr; ++rg) {
            const unsigned char* row = st + (size_t)rg * p.row_bytes;
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int v = v0 + lane + 32 * j;
                if (v < v1) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(row + (size_t)v * 16);
                    float wf[VEC];
                    unpack16<W>(wv, wf);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc = fmaf(xr[j][e], wf[e], acc);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) part[(size_t)(c * p.rows_per_stage + rg) * NWC + warp] = acc;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (failed && lane == 0) {
        atomicOr(p.status, GT_STATUS_TIMEOUT);
        abort_s = 1;
    }
    // every consumer warp reaches this barrier, failed or not (no wait is left
    // unbounded); then all of them leave together when any gave up (the
    // producer drains the copies in flight)
    asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
    if (ks > 1) {
        // split-K: rank 0 sums the cluster's partials (rank order, then warp
        // order) and applies the epilogue; the second barrier keeps every
        // rank's shared memory alive until rank 0 has read it
        cluster_sync_all();
        if (krank == 0 && !*(volatile int*)&abort_s) {
            for (int u = tid; u < nrows; u += NWC * 32) {
                float s2 = 0.f;
                for (int kr = 0; kr < ks; ++kr)
                    for (int w2 = 0; w2 < NWC; ++w2) s2 += ld_cluster_f32(part + (size_t)u * NWC + w2, (uint32_t)kr);
                if (YM == Y_RESID) p.y[r0 + u] = __ldcg(p.y + r0 + u) + s2;
                else if (YM == Y_PUSH) push_row(p, r0 + u, s2);
                else p.y[r0 + u] = s2;
            }
        }
        cluster_sync_all();
        return;
    }
    if (*(volatile int*)&abort_s) return;

    // ---- epilogue: fixed-order sum of the warp partials of every row
    for (int u = tid; u < nrows / RU; u += NWC * 32) {
        if (YM == Y_SWIGLU) {
            float g = 0.f, up = 0.f;
            for (int w2 = 0; w2 < NWC; ++w2) {
                g += part[(size_t)(2 * u) * NWC + w2];
                up += part[(size_t)(2 * u + 1) * NWC + w2];
            }
            p.y[(r0 >> 1) + u] = silu(g) * up;  // src/models/qwen3/module.cpp:466-468
        } else {
            float s2 = 0.f;
            for (int w2 = 0; w2 < NWC; ++w2) s2 += part[(size_t)u * NWC + w2];
            if (YM == Y_RESID) p.y[r0 + u] = __ldcg(p.y + r0 + u) + s2;  // src/models/qwen3/module.cpp:238-240
            else if (YM == Y_PUSH) push_row(p, r0 + u, s2);
            else p.y[r0 + u] = s2;
        }
    }
}

// Grouped expert down projection + weighted residual (MoE, batch 1), fed by
// TMA bulk copies: x[j] += sum over slots s in order of w_s * (W_down[ids[s]]
// row j . h_s) (src/models/qwen3/module.cpp:469-474, one expert at a time).
//
// A CTA owns a contiguous range of output rows j; a ring stage holds the same
// R rows of every selected expert ([slot][R rows], one copy per slot). Eight
// consumer warps: warp s computes slot s's dot products over the whole K (its
// lanes hold slot s's h vector in registers); the epilogue adds the slots in
// order into the residual. The ids come from the router, so the producer
// copies only after the dependency wait.
struct MoeDownTmaParams {
    const char* w;                     // [E][rows][K] expert matrices
    unsigned long long row_bytes;      // K * sizeof(W)
    unsigned long long expert_bytes;   // rows * row_bytes
    int rows;                          // d_model
    int K;                             // d_ff
    int k;                             // slots (1..8)
    const float* h;                    // [k][K]
    const int* ids;                    // [k]
    const float* ew;                   // [k]
    float* x;                          // [rows] residual, updated in place
    int rows_per_stage;                // output rows per stage
    int stages;
    uint32_t stage_bytes;              // k * rows_per_stage * row_bytes
    int* status;
    unsigned long long timeout_ns;
    // 1: the ids are read before the dependency wait, so the weight copies
    // overlap the previous kernel. Only for a previous kernel that let its
    // dependents launch after it had waited for the router (the grouped
    // gate/up GEMV does), so the router's ids are complete here.
    int ids_early;
    // expert parallelism: experts [ep_lo, ep_lo + ep_n) are stored here
    // (ep_n == 0: all). With push, this rank's slots are summed from zero in
    // slot order and the partial row is sent as tagged words to every rank's
    // receive slot of exchange ar_seq (the next layer's receive adds the
    // ranks' partials to the residual); x is then not touched.
    int ep_lo, ep_n;
    int push;
    CommDev comm;
    int ar_seq;
    const int* step;
};

constexpr int MD_WARPS = 8;  // consumer warps = the most slots
MF_DEVICE bool md_local(const MoeDownTmaParams& p, int e) { return p.ep_n == 0 || (e >= p.ep_lo && e < p.ep_lo + p.ep_n); }

template <typename W, int J>
__global__ void __launch_bounds__((MD_WARPS + 1) * 32, 1) moe_down_tma_kernel(const MoeDownTmaParams p) {
    constexpr int VEC = W::VEC;
    extern __shared__ __align__(128) unsigned char gt_smem[];
    __shared__ __align__(8) uint64_t full[GT_MAX_STAGES], empty[GT_MAX_STAGES];
    __shared__ int eid_s[MD_WARPS];
    __shared__ int abort_s;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r0 = (int)((long long)blockIdx.x * p.rows / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * p.rows / gridDim.x);
    const int nrows = r1 - r0, R = p.rows_per_stage, S = p.stages;
    const int nchunks = (nrows + R - 1) / R;
    float* ys = reinterpret_cast<float*>(gt_smem + (size_t)S * p.stage_bytes);  // [k][nrows]

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MD_WARPS);
        }
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned long long deadline = globaltimer_ns() + p.timeout_ns;

    if (warp == MD_WARPS) {
        pdl_launch_dependents();
        if (lane == 0) {
            if (!p.ids_early) pdl_wait();
            uint32_t n_loc = 0;
            for (int i = 0; i < p.k; ++i) {
                eid_s[i] = __ldcg(p.ids + i);  // from L2: written by the router
                n_loc += md_local(p, eid_s[i]) ? 1u : 0u;
            }
            const int ebase = p.ep_n ? p.ep_lo : 0;
            bool failed = false;
            int c = 0;
            for (; c < nchunks; ++c) {
                const int s = c % S;
                if (c >= S && !mbar_wait(&empty[s], (uint32_t)((c / S - 1) & 1), deadline, failed)) break;
                if (*(volatile int*)&abort_s) break;
                const int rr = min(R, nrows - c * R);
                const uint32_t bytes = (uint32_t)(rr * p.row_bytes);
                mbar_expect_tx(&full[s], bytes * n_loc);
                for (int sl = 0; sl < p.k; ++sl)
                    if (md_local(p, eid_s[sl]))
                        bulk_load(gt_smem + (size_t)s * p.stage_bytes + (size_t)sl * R * p.row_bytes,
                                  p.w + (size_t)(eid_s[sl] - ebase) * p.expert_bytes +
                                      (size_t)(r0 + c * R) * p.row_bytes,
                                  bytes, &full[s]);
            }
            if (failed) {
                atomicOr(p.status, GT_STATUS_TIMEOUT);
                abort_s = 1;
            }
            bool drain_failed = false;
            for (int d = max(0, c - S); d < c; ++d)
                mbar_wait(&full[d % S], (uint32_t)((d / S) & 1), deadline + p.timeout_ns, drain_failed);
        }
        return;
    }

    // ---- consumer warp `warp` = slot `warp` (warps past k, and slots whose
    // expert is stored on another rank, only release stages)
    const int NV = p.K / VEC;
    float xr[J][VEC];
    pdl_launch_dependents();
    pdl_wait();
    const bool active = warp < p.k && md_local(p, __ldcg(p.ids + warp));
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int v = lane + 32 * j;
#pragma unroll
        for (int e = 0; e < VEC; e += 4) {
            float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
            if (active && v < NV) t = __ldcg(reinterpret_cast<const float4*>(p.h + (size_t)warp * p.K + (size_t)v * VEC + e));
            xr[j][e] = t.x; xr[j][e + 1] = t.y; xr[j][e + 2] = t.z; xr[j][e + 3] = t.w;
        }
    }
    bool failed = false;
    for (int c = 0; c < nchunks; ++c) {
        const int s = c % S;
        if (!mbar_wait(&full[s], (uint32_t)((c / S) & 1), deadline, failed)) break;
        if (active) {
            const unsigned char* st = gt_smem + (size_t)s * p.stage_bytes + (size_t)warp * R * p.row_bytes;
            const int rr = min(R, nrows - c * R);
            int rg = 0;
            for (; rg + GT_RG <= rr; rg += GT_RG) {
                uint4 wv[GT_RG][J];
#pragma unroll
                for (int r = 0; r < GT_RG; ++r)
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        const int v = lane + 32 * j;
                        wv[r][j] = v < NV ? *reinterpret_cast<const uint4*>(st + (size_t)(rg + r) * p.row_bytes + (size_t)v * 16)
                                          : make_uint4(0u, 0u, 0u, 0u);
                    }
                float acc[GT_RG];
#pragma unroll
                for (int r = 0; r < GT_RG; ++r) {
                    acc[r] = 0.f;
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        float wf[VEC];
                        unpack16<W>(wv[r][j], wf);
#pragma unroll
                        for (int e = 0; e < VEC; ++e) acc[r] = fmaf(xr[j][e], wf[e], acc[r]);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int r = 0; r < GT_RG; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
                if (lane < GT_RG) {
                    float a = acc[0];
#pragma unroll
                    for (int r = 1; r < GT_RG; ++r)
                        if (lane == r) a = acc[r];
                    ys[(size_t)warp * nrows + c * R + rg + lane] = a;
                }
            }
            for (; rg < rr; ++rg) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int v = lane + 32 * j;
                    if (v < NV) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(st + (size_t)rg * p.row_bytes + (size_t)v * 16);
                        float wf[VEC];
                        unpack16<W>(wv, wf);
#pragma unroll
                        for (int e = 0; e < VEC; ++e) acc = fmaf(xr[j][e], wf[e], acc);
                    }
                }
                acc = warp_sum(acc);
                if (lane == 0) ys[(size_t)warp * nrows + c * R + rg] = acc;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (failed && lane == 0) {
        atomicOr(p.status, GT_STATUS_TIMEOUT);
        abort_s = 1;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(MD_WARPS * 32) : "memory");
    if (*(volatile int*)&abort_s) return;
    // src/models/qwen3/module.cpp:471-474: x += expert_out * weight, one expert at a time
    if (p.push) {
        // this rank's slots only, in slot order, from zero; the receiver adds
        // the ranks' partials to the residual in rank order
        const uint32_t tag = comm_tag(__ldcg(p.step + MF_STEP_FRAME), p.ar_seq);
        for (int u = tid; u < nrows; u += MD_WARPS * 32) {
            float part = 0.f;
            for (int sl = 0; sl < p.k; ++sl)
                if (md_local(p, __ldcg(p.ids + sl))) part = fmaf(ys[(size_t)sl * nrows + u], __ldcg(p.ew + sl), part);
            const unsigned long long w = tagged(part, tag);
            for (int r = 0; r < p.comm.tp_size; ++r) st_tagged(p.comm.recv(r, p.ar_seq & 1, p.comm.tp_rank) + r0 + u, w);
        }
        return;
    }
    for (int u = tid; u < nrows; u += MD_WARPS * 32) {
        float xo = __ldcg(p.x + r0 + u);
        for (int sl = 0; sl < p.k; ++sl) xo = fmaf(ys[(size_t)sl * nrows + u], __ldcg(p.ew + sl), xo);
        p.x[r0 + u] = xo;
    }
}

}  // namespace mf

namespace mf {
// Kernel pointer for (dtype, x mode, y mode, consumer warps, J); null when not built.
template <typename W>
const void* gemv_tma_ptr(int xm, int ym, int nwc, int j) {
#define MF_GT(NW, JJ)                                                                                        \
    if (nwc == NW && j == JJ) {                                                                              \
        if (xm == X_NORM && ym == Y_STORE) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_NORM, Y_STORE>; \
        if (xm == X_PLAIN && ym == Y_STORE) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_PLAIN, Y_STORE>; \
        if (xm == X_PLAIN && ym == Y_RESID) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_PLAIN, Y_RESID>; \
        if (xm == X_NORM && ym == Y_SWIGLU) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_NORM, Y_SWIGLU>; \
        if (xm == X_AR_NORM && ym == Y_STORE) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_AR_NORM, Y_STORE>; \
        if (xm == X_AR_NORM && ym == Y_SWIGLU)                                                                \
            return (const void*)&gemv_tma_kernel<W, NW, JJ, X_AR_NORM, Y_SWIGLU>;                            \
        if (xm == X_PLAIN && ym == Y_PUSH) return (const void*)&gemv_tma_kernel<W, NW, JJ, X_PLAIN, Y_PUSH>; \
        return nullptr;                                                                                       \
    }
    MF_GT(8, 1)
    MF_GT(8, 2)
    MF_GT(8, 3)
    MF_GT(8, 4)
    MF_GT(8, 6)
    MF_GT(8, 8)
    MF_GT(16, 8)
#undef MF_GT
    return nullptr;
}
template <typename W>
const void* moe_down_tma_ptr(int j) {
    switch (j) {
        case 1: return (const void*)&moe_down_tma_kernel<W, 1>;
        case 2: return (const void*)&moe_down_tma_kernel<W, 2>;
        case 3: return (const void*)&moe_down_tma_kernel<W, 3>;
        case 4: return (const void*)&moe_down_tma_kernel<W, 4>;
        case 6: return (const void*)&moe_down_tma_kernel<W, 6>;
        case 8: return (const void*)&moe_down_tma_kernel<W, 8>;
        default: return nullptr;
    }
}
const void* gemv_tma_ptr_f32(int xm, int ym, int nwc, int j);
const void* gemv_tma_ptr_f16(int xm, int ym, int nwc, int j);
const void* gemv_tma_ptr_bf16(int xm, int ym, int nwc, int j);
const void* moe_down_tma_ptr_f32(int j);
const void* moe_down_tma_ptr_f16(int j);
const void* moe_down_tma_ptr_bf16(int j);
}  // namespace mf
