// Decode GEMV family: y = W x for one fp32 activation vector, W streamed from
// HBM once per token.
//
// What it computes follows the reference's matmul_{fp32,fp16,bf16}
// (src/ops/kernels.cpp:211-343): weights widened to fp32, fp32 FMAs, fp32
// result per row. The summation order differs (the reference keeps 16 NEON
// lanes per row; here a CTA splits each row over its threads), so results
// agree to fp32 rounding, not bitwise.
//
// Structure (B200):
//  * A CTA owns a contiguous, balanced range of "units" (rows, gate/up row
//    pairs, or output rows of a grouped expert product), so per-SM bytes are
//    equal to within one unit.
//  * All T threads of a CTA span the K axis: thread t reads 16-byte vectors at
//    columns (pass*T + t)*VEC. A tile of R rows is read PC passes at a time,
//    so every thread keeps R*PC = 8 independent 16-byte loads in flight, and
//    the next step's loads are issued before the current step is reduced
//    (two register buffers).
//  * The activation vector lives in shared memory (optionally RMS-normalised
//    in the prologue, which fuses the reference's separate rmsnorm pass; the
//    norm weights are staged before the dependency wait, x is read once).
//  * Programmatic dependent launch: dense weight loads are issued before
//    griddepcontrol.wait, so they overlap the previous kernel's tail.
//    Everything written by earlier kernels is read through L2 (ld.cg).
#pragma once

#include "comm.cuh"
#include "mf_common.cuh"

namespace mf {

// X_AR_NORM: the activation is the residual plus every tensor-parallel rank's
// partial vector of an all-reduce (waited for in the prologue), then RMSNorm.
// Y_PUSH: the rows' partial sums are stored into every rank's receive slot of
// an all-reduce instead of locally.
enum XMode { X_PLAIN = 0, X_NORM = 1, X_AR_NORM = 2 };
// Y_MOE_PUSH: the grouped expert down projection of this rank's experts,
// pushed as its partial of an all-reduce (expert parallelism).
enum YMode { Y_STORE = 0, Y_RESID = 1, Y_SWIGLU = 2, Y_MOE_DOWN = 3, Y_PUSH = 4, Y_MOE_PUSH = 5 };

struct GemvParams {
    const void* w;        // weight rows, dtype given by the template
    size_t w_offset;      // element offset added to w (reference `offset` argument)
    const float* x;       // activation vector(s)
    const float* nw;      // RMSNorm weight for X_NORM
    float eps;
    float* y;             // output
    int rows;             // logical rows (Y_MOE_DOWN: output rows)
    int K;                // row length (elements)
    // expert indirection (Y_SWIGLU over experts, Y_MOE_DOWN)
    const int* expert_ids;      // [k] device, or null for dense weights
    const float* expert_w;      // [k] device (Y_MOE_DOWN)
    int rows_per_expert;        // physical rows per expert matrix
    int n_slots;                // k for Y_MOE_DOWN / Y_MOE_PUSH
    // expert parallelism: only experts [ep_lo, ep_lo + ep_n) are stored here
    // (expert e at local index e - ep_lo); slots routed elsewhere contribute
    // nothing. ep_n == 0: every expert is local.
    int ep_lo, ep_n;
    // greedy argmax finisher (Y_STORE only; counter may be null)
    float* best_val;            // [gridDim.x]
    int* best_idx;              // [gridDim.x]
    int* counter;               // zero-initialised; reset by the last CTA
    int* step;                  // device step record {token, pos, next_token, chain}
    int vocab_offset;           // index of row 0 (vocab-split lm_head)
    int pf_tiles;               // L2 prefetch depth in tiles (tiles <= 48 KB)
    // tensor parallelism (X_AR_NORM, Y_PUSH, and the lm_head's cross-rank argmax)
    CommDev comm;
    int ar_seq;                 // exchange number within the frame (slot = ar_seq & 1); tag from step[frame]
    const float* x_res;         // X_AR_NORM: residual before the all-reduce
    float* x_out;               // X_AR_NORM: residual after it (written by CTA 0)
    int gather_logits;          // Y_STORE + TP: also store rows into every rank's full-logits buffer
};

#ifndef MF_GEMV_MIN_BLOCKS
#define MF_GEMV_MIN_BLOCKS 1
#endif

// The all-reduce receive prologue holds tagged words next to the first
// weight loads: keep such kernels at two resident CTAs per SM.
MF_DEVICE bool expert_local(const GemvParams& p, int e) { return p.ep_n == 0 || (e >= p.ep_lo && e < p.ep_lo + p.ep_n); }

template <typename W, int T, int R, int PC, int XM, int YM>
__global__ void __launch_bounds__(T, (XM == X_AR_NORM && MF_GEMV_MIN_BLOCKS < 2) ? 2 : MF_GEMV_MIN_BLOCKS)
    gemv_kernel(const GemvParams p) {
    constexpr bool MOE_DOWN = (YM == Y_MOE_DOWN || YM == Y_MOE_PUSH);
    constexpr int VEC = W::VEC;
    constexpr int NW = T / 32;
    constexpr int RU = (YM == Y_SWIGLU) ? 2 : 1;  // rows per unit
    static_assert(R * PC == 8, "8 loads in flight per thread");
    static_assert(YM != Y_SWIGLU || R % 2 == 0, "gate/up pairs");
    static_assert(R <= 32, "tile rows fit one warp");
    extern __shared__ float4 smem_f4[];
    float* xs = reinterpret_cast<float*>(smem_f4);
    __shared__ float red[2][NW][R];
    __shared__ float scratch[32];
    __shared__ int scratch_i[32];
    __shared__ int ids_s[32];    // expert ids of the slots (indirect modes), read once per launch
    __shared__ float ew_s[32];   // their routing weights (grouped down projection)
    __shared__ float cta_best_v;
    __shared__ int cta_best_i;
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.K;
    constexpr size_t esz = sizeof(typename W::T);
    const char* wbase = reinterpret_cast<const char*>(p.w) + p.w_offset * esz;
    const size_t row_bytes = (size_t)K * esz;

    // ---- unit range of this CTA
    const long long units = MOE_DOWN ? p.rows : p.rows / RU;
    const long long u0 = (long long)blockIdx.x * units / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * units / gridDim.x;
    const int rows0 = (int)(u0 * RU), rows1 = (int)(u1 * RU);
    // Y_MOE_DOWN: one output row per tile, tile row r = expert slot r.
    const int ntiles = MOE_DOWN ? (rows1 - rows0) : (rows1 - rows0 + R - 1) / R;
    constexpr int STEP_COLS = PC * T * VEC;
    const int nsteps = (K + STEP_COLS - 1) / STEP_COLS;
    const int nitems = ntiles * nsteps;
    const bool indirect = MOE_DOWN || (p.expert_ids != nullptr);
    const int n_ids = MOE_DOWN ? p.n_slots : (indirect ? p.rows / p.rows_per_expert : 0);
    const int ep_base = p.ep_n ? p.ep_lo : 0;
    // rows of the gate/up expert tile starting at logical row r0 lie in one
    // local expert: its first physical row (or -1 when not, or when the
    // slot's expert is stored on another rank)
    auto expert_tile_row = [&](int r0) -> long long {
        const int s0 = r0 / p.rows_per_expert;
        if ((min(r0 + R, rows1) - 1) / p.rows_per_expert != s0) return -1;
        const int e = ids_s[s0];
        if (!expert_local(p, e)) return -1;
        return (long long)(e - ep_base) * p.rows_per_expert + (r0 - s0 * p.rows_per_expert);
    };

    int eid[R];
#pragma unroll
    for (int r = 0; r < R; ++r) eid[r] = 0;

    constexpr size_t CSTRIDE = (size_t)T * VEC * esz;  // bytes between a thread's passes
    const bool k_exact = (K % STEP_COLS) == 0;
    auto load = [&](uint4 (&buf)[R][PC], int it) {
        const int tile = it / nsteps, step = it - tile * nsteps;
        const size_t coff = ((size_t)(step * PC) * T + tid) * VEC * esz;
        if (!indirect) {
            const int r0 = rows0 + tile * R;
            const char* tp = wbase + (size_t)r0 * row_bytes + coff;
            if (k_exact && r0 + R <= rows1) {
                // full tile: every lane loads, addresses are base + constants
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int c = 0; c < PC; ++c) buf[r][c] = ld_stream(tp + r * row_bytes + c * CSTRIDE);
                return;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int c = 0; c < PC; ++c) {
                    const int col = ((step * PC + c) * T + tid) * VEC;
                    if (r0 + r < rows1 && col < K) buf[r][c] = ld_stream(tp + r * row_bytes + c * CSTRIDE);
                    else buf[r][c] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            return;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            bool valid;
            long long phys;
            if (MOE_DOWN) {
                const int j = rows0 + tile;
                valid = r < p.n_slots && expert_local(p, eid[r]);
                phys = (long long)(eid[r] - (p.ep_n ? p.ep_lo : 0)) * p.rows_per_expert + j;
            } else {
                const int lr = rows0 + tile * R + r;
                valid = lr < rows1;
                const int slot = valid ? lr / p.rows_per_expert : 0;
                const int e = ids_s[slot];
                valid = valid && expert_local(p, e);
                phys = valid ? (long long)(e - ep_base) * p.rows_per_expert + (lr - slot * p.rows_per_expert) : 0;
            }
            const char* rp = wbase + phys * row_bytes + coff;
#pragma unroll
            for (int c = 0; c < PC; ++c) {
                const int col = ((step * PC + c) * T + tid) * VEC;
                if (valid && col < K) buf[r][c] = ld_stream(rp + c * CSTRIDE);
                else buf[r][c] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    // gate/up over experts: a full tile inside one local expert is a
    // contiguous run of rows, loaded like a dense tile
    auto load_expert = [&](uint4 (&buf)[R][PC], int it) {
        if (!MOE_DOWN && k_exact) {
            const int tile = it / nsteps, step = it - tile * nsteps;
            const int r0 = rows0 + tile * R;
            const long long pr = (r0 + R <= rows1) ? expert_tile_row(r0) : -1;
            if (pr >= 0) {
                const size_t coff = ((size_t)(step * PC) * T + tid) * VEC * esz;
                const char* tp = wbase + (size_t)pr * row_bytes + coff;
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int c = 0; c < PC; ++c) buf[r][c] = ld_stream(tp + r * row_bytes + c * CSTRIDE);
                return;
            }
        }
        load(buf, it);
    };

    // L2 prefetch window (dense weights): the CTA's rows are one contiguous
    // byte range, so one bulk prefetch per tile keeps `pf_ahead` tiles in
    // flight ahead of the register loads without holding registers.
    const size_t tile_bytes = (size_t)R * row_bytes;
    const int pf_ahead = MOE_DOWN ? -1
                                  : (tile_bytes <= 48 * 1024 ? p.pf_tiles : (tile_bytes <= 128 * 1024 ? 1 : -1));
    auto prefetch_tile = [&](int t) {
        if (t >= ntiles) return;
        const int r0 = rows0 + t * R;
        const int r1 = min(r0 + R, rows1);
        if (indirect) {
            const long long pr = expert_tile_row(r0);
            if (pr >= 0) prefetch_l2(wbase + (size_t)pr * row_bytes, (uint32_t)((size_t)(r1 - r0) * row_bytes));
            return;
        }
        prefetch_l2(wbase + (size_t)r0 * row_bytes, (uint32_t)((size_t)(r1 - r0) * row_bytes));
    };

    uint4 bufA[R][PC], bufB[R][PC];
    // Dense weights and norm weights do not depend on earlier kernels: start
    // streaming them before the dependency wait. Expert ids come from the
    // router kernel.
    if (tid == 0 && !indirect)
        for (int t = 0; t <= pf_ahead; ++t) prefetch_tile(t);
    if (!indirect && nitems > 0) load(bufA, 0);
    if (XM == X_NORM || XM == X_AR_NORM)
        for (int i = tid; i < K; i += T) xs[K + i] = __ldg(p.nw + i);
    // Triggering this early lets the next kernel's CTAs become resident and
    // start their own weight loads while this one runs (measured faster than
    // triggering after the last weight load).
    pdl_launch_dependents();
    pdl_wait();
    if (indirect) {
        // expert ids (and weights) come from the router kernel: read them once
        if (tid < 32) {
            ids_s[tid] = tid < n_ids ? __ldcg(p.expert_ids + tid) : 0;
            ew_s[tid] = (MOE_DOWN && tid < n_ids) ? __ldcg(p.expert_w + tid) : 0.f;
        }
        __syncthreads();
        if (MOE_DOWN) {
#pragma unroll
            for (int r = 0; r < R; ++r) eid[r] = (r < p.n_slots) ? ids_s[r] : 0;
        }
        if (tid == 0)
            for (int t = 0; t <= pf_ahead; ++t) prefetch_tile(t);
        if (nitems > 0) load_expert(bufA, 0);
    }

    // tagged words of a push (tensor-parallel send)
    uint32_t push_tag = 0;
    if (YM == Y_PUSH || YM == Y_MOE_PUSH) push_tag = comm_tag(__ldcg(p.step + MF_STEP_FRAME), p.ar_seq);

    // ---- prologue: activation vector(s) -> shared memory
    if (XM == X_NORM || XM == X_AR_NORM) {
        float ss = 0.f;
        if (XM == X_AR_NORM) {
            // all-reduce receive: x = residual + partial_0 + partial_1 + ...
            // in rank order (identical on every rank), each partial element
            // read once its tag shows it is this exchange's. Each CTA reduces
            // only its slice of x into x_out; after a grid barrier every CTA
            // reads the whole reduced x_out (the partials cross L2 once, not
            // once per CTA).
            const uint32_t tag = comm_tag(__ldcg(p.step + MF_STEP_FRAME), p.ar_seq);
            const int slot = p.ar_seq & 1;
            int* status = &p.comm.local()->status;
            const unsigned long long deadline = globaltimer_ns() + p.comm.timeout_ns;
            bool late = false;
            const int e0 = (int)((long long)blockIdx.x * K / gridDim.x);
            const int e1 = (int)((long long)(blockIdx.x + 1) * K / gridDim.x);
            recv_sum(p.comm, slot, tag, p.x_res, e0 + tid, T, e1, deadline, &late, status,
                     [&](int i, float v) { p.x_out[i] = v; });
            __threadfence();
            __syncthreads();
            if (tid == 0)
                grid_arrive_wait(&p.comm.local()->bar[slot], tag, gridDim.x, deadline, &late, status,
                                 COMM_STATUS_AR_TIMEOUT);
            __syncthreads();
            for (int i = tid * 4; i < K; i += T * 4) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(p.x_out + i));
                *reinterpret_cast<float4*>(xs + i) = v;
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
        } else {
            for (int i = tid; i < K; i += T) {
                const float v = __ldcg(p.x + i);
                xs[i] = v;
                ss = fmaf(v, v, ss);
            }
        }
        ss = block_sum(ss, scratch);  // (its barrier also publishes every thread's xs stores)
        // src/ops/kernels.cpp:355-363: rms = sqrtf(ss/dim + eps); inv = 1/rms; out = inv*x*w
        // (each thread rescales the elements it stored itself)
        const float inv = 1.0f / sqrtf(ss / (float)K + p.eps);
        for (int i = tid; i < K; i += T) xs[i] = (inv * xs[i]) * xs[K + i];
    } else {
        // all of a thread's 16-byte loads of a batch are issued before any is stored
        const int xlen = MOE_DOWN ? K * p.n_slots : K;
        constexpr int XB = 8;
        for (int i0 = tid * 4; i0 < xlen; i0 += T * 4 * XB) {
            float4 v[XB];
#pragma unroll
            for (int u = 0; u < XB; ++u) {
                const int i = i0 + u * T * 4;
                if (i < xlen) v[u] = __ldcg(reinterpret_cast<const float4*>(p.x + i));
            }
#pragma unroll
            for (int u = 0; u < XB; ++u) {
                const int i = i0 + u * T * 4;
                if (i < xlen) *reinterpret_cast<float4*>(xs + i) = v[u];
            }
        }
    }
    if (tid == 0) {
        cta_best_v = -INFINITY;
        cta_best_i = 0x7fffffff;
    }
    __syncthreads();

    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    int par = 0;

    float y_pre = 0.f;  // Y_MOE_DOWN: the residual of the tile's output row, fetched early
    auto consume = [&](const uint4 (&buf)[R][PC], int it) {
        const int tile = it / nsteps, step = it - tile * nsteps;
        if (YM == Y_MOE_DOWN && step == 0 && tid == 0) y_pre = __ldcg(p.y + rows0 + tile);
#pragma unroll
        for (int c = 0; c < PC; ++c) {
            const int col = ((step * PC + c) * T + tid) * VEC;
            if (col < K) {
                if (MOE_DOWN) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (r >= p.n_slots) break;  // xs holds n_slots vectors only
                        float wv[VEC];
                        unpack16<W>(buf[r][c], wv);
                        const float* xr = xs + r * K + col;
#pragma unroll
                        for (int e = 0; e < VEC; e += 4) {
                            const float4 t4 = *reinterpret_cast<const float4*>(xr + e);
                            acc[r] = fmaf(t4.x, wv[e], acc[r]);
                            acc[r] = fmaf(t4.y, wv[e + 1], acc[r]);
                            acc[r] = fmaf(t4.z, wv[e + 2], acc[r]);
                            acc[r] = fmaf(t4.w, wv[e + 3], acc[r]);
                        }
                    }
                } else {
                    float xv[VEC];
#pragma unroll
                    for (int e = 0; e < VEC; e += 4) {
                        const float4 t4 = *reinterpret_cast<const float4*>(xs + col + e);
                        xv[e] = t4.x; xv[e + 1] = t4.y; xv[e + 2] = t4.z; xv[e + 3] = t4.w;
                    }
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float wv[VEC];
                        unpack16<W>(buf[r][c], wv);
#pragma unroll
                        for (int e = 0; e < VEC; ++e) acc[r] = fmaf(xv[e], wv[e], acc[r]);
                    }
                }
            }
        }
        if (step != nsteps - 1) return;
        // ---- tile complete: CTA-wide reduction in a fixed order
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float v = warp_sum(acc[r]);
            if (lane == 0) red[par][warp][r] = v;
            acc[r] = 0.f;
        }
        __syncthreads();
        if (warp == 0) {
            if (YM == Y_MOE_DOWN) {
                if (lane == 0) {
                    const int j = rows0 + tile;
                    // src/models/qwen3/module.cpp:471-474: x += expert_out * weight, one expert at a time
                    float xo = y_pre;
                    for (int r = 0; r < p.n_slots; ++r) {
                        float s = 0.f;
                        for (int w2 = 0; w2 < NW; ++w2) s += red[par][w2][r];
                        xo = fmaf(s, ew_s[r], xo);
                    }
                    p.y[j] = xo;
                }
            } else if (YM == Y_MOE_PUSH) {
                if (lane == 0) {
                    // this rank's experts only, in slot order; the receiver adds
                    // the ranks' partials to the residual in rank order
                    const int j = rows0 + tile;
                    float part = 0.f;
                    for (int r = 0; r < p.n_slots; ++r) {
                        if (!expert_local(p, eid[r])) continue;
                        float s = 0.f;
                        for (int w2 = 0; w2 < NW; ++w2) s += red[par][w2][r];
                        part = fmaf(s, ew_s[r], part);
                    }
                    const unsigned long long w = tagged(part, push_tag);
                    for (int r = 0; r < p.comm.tp_size; ++r)
                        st_tagged(p.comm.recv(r, p.ar_seq & 1, p.comm.tp_rank) + j, w);
                }
            } else if (YM == Y_SWIGLU) {
                const int lr = rows0 + tile * R + 2 * lane;
                if (lane < R / 2 && lr < rows1) {
                    float g = 0.f, u = 0.f;
                    for (int w2 = 0; w2 < NW; ++w2) {
                        g += red[par][w2][2 * lane];
                        u += red[par][w2][2 * lane + 1];
                    }
                    // src/models/qwen3/module.cpp:466-468: h = silu(g) * u
                    p.y[lr / 2] = silu(g) * u;
                }
            } else {
                const int lr = rows0 + tile * R + lane;
                const bool valid = lane < R && lr < rows1;
                float s = 0.f;
                if (valid) {
                    for (int w2 = 0; w2 < NW; ++w2) s += red[par][w2][lane];
                    if (YM == Y_RESID) {
                        p.y[lr] = __ldcg(p.y + lr) + s;  // src/models/qwen3/module.cpp:238-240
                    } else if (YM == Y_PUSH) {
                        const unsigned long long w = tagged(s, push_tag);
                        for (int r = 0; r < p.comm.tp_size; ++r)
                            st_tagged(p.comm.recv(r, p.ar_seq & 1, p.comm.tp_rank) + lr, w);
                    } else {
                        p.y[lr] = s;
                        if (YM == Y_STORE && p.gather_logits)
                            for (int r = 0; r < p.comm.tp_size; ++r) p.comm.gather(r)[p.vocab_offset + lr] = s;
                    }
                }
                if (YM == Y_STORE && p.counter != nullptr) {
                    float bv = valid ? s : -INFINITY;
                    int bi = valid ? p.vocab_offset + lr : 0x7fffffff;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                    }
                    if (lane == 0 && better(bv, bi, cta_best_v, cta_best_i)) {
                        cta_best_v = bv;
                        cta_best_i = bi;
                    }
                }
            }
        }
        par ^= 1;
    };

    auto advance_prefetch = [&](int it) {
        if (pf_ahead >= 0 && tid == 0 && it % nsteps == 0) prefetch_tile(it / nsteps + pf_ahead + 1);
    };
    auto load_any = [&](uint4 (&buf)[R][PC], int it) {
        if (indirect) load_expert(buf, it);
        else load(buf, it);
    };
#ifdef MF_GEMV_SINGLE_BUFFER
    for (int it = 0; it < nitems; ++it) {
        advance_prefetch(it);
        if (it > 0) load_any(bufA, it);
        consume(bufA, it);
    }
#else
    for (int it = 0; it < nitems; it += 2) {
        advance_prefetch(it);
        if (it + 1 < nitems) load_any(bufB, it + 1);
        consume(bufA, it);
        if (it + 1 >= nitems) break;
        advance_prefetch(it + 1);
        if (it + 2 < nitems) load_any(bufA, it + 2);
        consume(bufB, it + 1);
    }
#endif

    // ---- greedy argmax finisher: the last CTA reduces the per-CTA candidates
    if (YM == Y_STORE && p.counter != nullptr) {
        if (p.gather_logits && warp == 0) __threadfence_system();  // logits rows stored on peers
        __syncthreads();
        if (tid == 0) {
            p.best_val[blockIdx.x] = cta_best_v;
            p.best_idx[blockIdx.x] = cta_best_i;
            __threadfence();
            const int ticket = atomicAdd(p.counter, 1);
            is_last = (ticket == (int)gridDim.x - 1);
        }
        __syncthreads();
        if (is_last) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int b = tid; b < (int)gridDim.x; b += T) {
                const float v = __ldcg(p.best_val + b);
                const int i = __ldcg(p.best_idx + b);
                if (better(v, i, bv, bi)) { bv = v; bi = i; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) {
                scratch[warp] = bv;
                scratch_i[warp] = bi;
            }
            __syncthreads();
            if (tid == 0) {
                float fv = scratch[0];
                int fi = scratch_i[0];
                for (int w2 = 1; w2 < NW; ++w2) {
                    if (better(scratch[w2], scratch_i[w2], fv, fi)) { fv = scratch[w2]; fi = scratch_i[w2]; }
                }
                // no candidate (every logit NaN): std::max_element returns the first element
                if (fi == 0x7fffffff) fi = p.vocab_offset;
                if (p.comm.tp_size > 1) {
                    // vocab split over ranks: exchange the per-rank maxima as
                    // tagged words, then reduce them in rank order (every rank
                    // picks the same id). In gather mode every CTA fenced its
                    // logits stores before its ticket, so they are visible on
                    // the peers before this rank's maximum is.
                    const uint32_t tag = comm_tag(p.step[MF_STEP_FRAME], COMM_SEQ_GREEDY);
                    const unsigned long long wv = tagged(fv, tag), wi = tagged(__int_as_float(fi), tag);
                    for (int r = 0; r < p.comm.tp_size; ++r) {
                        st_tagged(p.comm.best(r) + 2 * p.comm.tp_rank, wv);
                        st_tagged(p.comm.best(r) + 2 * p.comm.tp_rank + 1, wi);
                    }
                    int* status = &p.comm.local()->status;
                    const unsigned long long deadline = globaltimer_ns() + p.comm.timeout_ns;
                    bool late = false;
                    const unsigned long long* b = p.comm.best(p.comm.tp_rank);
                    for (int r = 0; r < p.comm.tp_size; ++r) {
                        const float v = recv_tagged(b + 2 * r, tag, deadline, &late, status, COMM_STATUS_LM_TIMEOUT);
                        const int i = __float_as_int(
                            recv_tagged(b + 2 * r + 1, tag, deadline, &late, status, COMM_STATUS_LM_TIMEOUT));
                        if (r == 0 || better(v, i, fv, fi)) {
                            fv = v;
                            fi = i;
                        }
                    }
                    // every wait of this frame is behind us (earlier kernels, this
                    // kernel's CTAs before their tickets, the exchange above): the
                    // host reads the sticky status bits with the step record
                    p.step[MF_STEP_STATUS] = *(volatile int*)status;
                }
                // greedy id -> next_token; a chained record also becomes the
                // next step's input so decode can continue without the host
                p.step[2] = fi;
                if (p.step[3] != 0) {
                    p.step[0] = fi;
                    p.step[1] = p.step[1] + 1;
                    p.step[MF_STEP_FRAME] = p.step[MF_STEP_FRAME] + 1;
                }
                *p.counter = 0;
            }
        }
    }
}

}  // namespace mf
