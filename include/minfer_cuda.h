/*
 * minfer_cuda.h — C ABI of libmfcuda.so, the sm_100a (B200) device layer of the
 * Qwen3 token loop.
 *
 * It takes the place of two reference interfaces:
 *   - the Metal device manager, include/minfer/interfaces/metal_interface.hpp:9-37
 *     (MetalManager::init/upload/release/cpu_ptr/begin_frame/end_frame/dispatch*);
 *   - the name-addressed GPU kernels dispatched from src/models/qwen3/module.cpp
 *     (MetalManager::dispatch1d/2d("linear_proj_bf16", ...) and friends), which
 *     become typed entry points below.
 *
 * Conventions
 *   - Every entry point returns MF_OK (0) or a negative MF_E_* status; the
 *     message of the last failure on the calling thread is available through
 *     mf_last_error(). No C++ exception crosses this boundary.
 *   - Device buffers are plain device addresses (`void*`, `float*`), obtained
 *     from mf_upload/mf_alloc (mf_ptr) or from any other CUDA allocator.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the manager stream
 *     of the current device (mf_init must have been called).
 *   - Weight dtypes use the reference's DataType codes
 *     (include/minfer/base/types.hpp:5): MF_F32 = 0, MF_F16 = 1, MF_BF16 = 2.
 *   - Activations, KV cache, logits: fp32, as in the reference's RunState
 *     (include/minfer/base/config.hpp:77-102).
 *   - Not thread-safe, like the reference's process-global Metal context
 *     (src/interfaces/metal_interface.mm:59): drive a manager from one thread.
 */
#ifndef MINFER_CUDA_H
#define MINFER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define MF_OK 0
#define MF_E_INVALID (-1)     /* bad argument (null pointer, size, dtype, shape) */
#define MF_E_CUDA (-2)        /* a CUDA runtime call failed */
#define MF_E_OOM (-3)         /* device allocation failed or request too large */
#define MF_E_TIMEOUT (-4)     /* a bounded wait gave up (peer never arrived) */
#define MF_E_UNSUPPORTED (-5) /* shape/dtype combination without a kernel */
#define MF_E_STATE (-6)       /* call out of order (e.g. no mf_init) */
#define MF_E_IO (-7)          /* file could not be read or parsed */

/* ---- dtypes (reference DataType, include/minfer/base/types.hpp:5) ---- */
#define MF_F32 0
#define MF_F16 1
#define MF_BF16 2

/* ---- frames --------------------------------------------------------- */
#define MF_FRAME_RECORD 0 /* begin_frame: ops issued now are captured */
#define MF_FRAME_REPLAY 1 /* begin_frame: a captured frame exists; issue nothing */
#define MF_FRAME_NO_UPLOAD 1 /* begin_frame_ex flag: keep the device step record as is */

typedef struct mf_buf mf_buf;

/* ===================================================================== */
/* Manager — replaces MetalManager (metal_interface.hpp:9-37)             */
/* ===================================================================== */

/* MetalManager::init (src/interfaces/metal_interface.mm:81-109). Selects the
 * devices of `n_ranks` ranks (devices == NULL: 0..n_ranks-1) and creates one
 * stream per rank. Calling it again with the same arguments is a no-op. */
int mf_init(int n_ranks, const int* devices);
/* Releases every frame, stream and buffer still owned by the manager. */
int mf_shutdown(void);
/* Number of visible CUDA devices. */
int mf_device_count(int* count);
/* Message of the last failure on this thread (always NUL-terminated). */
int mf_last_error(char* buf, size_t n);

/* MetalManager::upload (metal_interface.mm:65-70): copy `bytes` from host
 * memory into a new device buffer of rank `rank`. */
int mf_upload(const void* host, size_t bytes, int rank, mf_buf** out);
/* Zero-filled device buffer of `bytes` on rank `rank`. */
int mf_alloc(size_t bytes, int rank, mf_buf** out);
/* MetalManager::release (metal_interface.mm:72-74). NULL is ignored. */
void mf_release(mf_buf* buf);
/* Device address of a buffer (the handle the ops take). */
void* mf_ptr(const mf_buf* buf);
size_t mf_size(const mf_buf* buf);
/* Explicit copies replace MetalManager::cpu_ptr's shared-memory view
 * (metal_interface.mm:76-78). Both synchronise the rank's stream. */
int mf_read(const mf_buf* buf, size_t offset, void* host, size_t bytes);
int mf_write(mf_buf* buf, size_t offset, const void* host, size_t bytes);

/* Strided upload: `rows` runs of `width` bytes from host (src_pitch apart)
 * into buf at offset, dst_pitch apart. Used to lay weights out for the
 * kernels (e.g. gate/up rows interleaved) straight from the mapped file. */
int mf_write_2d(mf_buf* buf, size_t offset, size_t dst_pitch, const void* host, size_t src_pitch, size_t width,
                size_t rows);
/* Device-to-device copy inside one rank's buffers (synchronous). */
int mf_copy(mf_buf* dst, size_t dst_off, const mf_buf* src, size_t src_off, size_t bytes);
/* Page-locked host memory (for per-token logits / ids). */
int mf_host_alloc(size_t bytes, void** out);
void mf_host_free(void* p);
/* Asynchronous device->host copy on `stream` (capturable inside a frame). */
int mf_copy_to_host_async(void* host, const void* dev, size_t bytes, void* stream);

/* MetalManager::begin_frame / end_frame (metal_interface.mm:111-137): one
 * frame is one token step. The first frame with a given id is captured into
 * a CUDA graph (returns MF_FRAME_RECORD: issue the ops now); later frames with
 * that id return MF_FRAME_REPLAY and the caller issues nothing. end_frame
 * launches the graph and waits for it, like the reference's commit+wait. */
int mf_begin_frame(int rank, int frame_id);
/* As begin_frame; with MF_FRAME_NO_UPLOAD the captured frame does not copy the
 * host step record in, so a chained record (see mf_lm_head) drives it. */
int mf_begin_frame_ex(int rank, int frame_id, int flags);
int mf_end_frame(int rank);
/* Same as end_frame without the wait (frames pipelined on the stream). */
int mf_end_frame_async(int rank);
/* Ends an open frame without launching it (a failed capture is discarded). */
int mf_abort_frame(int rank);
/* Drops every captured frame of `rank` (after buffers were reallocated). */
int mf_reset_frames(int rank);
/* Drops the captured frames of `rank` with ids in [first_id, last_id]. */
int mf_drop_frames(int rank, int first_id, int last_id);
/* Waits for all work on the rank's stream. */
int mf_sync(int rank);
/* The rank's stream as a cudaStream_t. */
void* mf_stream(int rank);
/* Device-side timing of everything issued on the rank's stream between
 * start and stop (CUDA events; stop waits for the stop event). */
int mf_timer_start(int rank);
int mf_timer_stop(int rank, float* ms);
/* Host-visible step record (MF_STEP_RECORD_BYTES) copied to the device at the
 * start of every frame launch: int32 {token, pos, next_token, chain, frame,
 * 0, 0, 0}. `frame` is a sequence number the caller advances for every frame
 * (a chained lm_head advances it on the device); the tensor-parallel
 * exchange tags its messages with it. Returns a pinned host pointer and the
 * matching device pointer. */
#define MF_STEP_RECORD_BYTES 32
#define MF_STEP_FRAME 4 /* index of the frame field */
#define MF_STEP_STATUS 5 /* exchange status bits (mf_comm_status), written by the tensor-parallel lm_head */
#define MF_STEP_DSTATUS 6 /* bit 1: a decode kernel's copy wait gave up (mf_decode_status) */
#define MF_STEP_SAMPLE 7  /* index of the next device-sampled token (mf_sample_step) */
int mf_step_state(int rank, int32_t** host, void** device);
/* Decode-kernel status of a rank (the MF_STEP_DSTATUS field of its device
 * step record, which the TMA-fed GEMVs set when a bounded copy wait gave up);
 * clear != 0 resets it. Synchronises the rank's stream. */
int mf_decode_status(int rank, int* status, int clear);

/* ===================================================================== */
/* Token-loop ops (fused). Each replaces a run of Metal dispatches of     */
/* src/models/qwen3/module.cpp; the cited lines are the CPU path they     */
/* reproduce.                                                             */
/* ===================================================================== */

/* Qwen3Embed (module.cpp:19-44): x[0:d) = fp32(emb[token]), token read from
 * the device step record (an id outside [0, vocab) reads row 0). */
int mf_embed_step(float* x, const void* emb, int dtype, int vocab, int d_model, const void* step_state,
                  void* stream);

/* Host helper: the NeoX RoPE (cos, sin) table, out[(p*(d_rot/2) + i)*2 + {0,1}]
 * for positions p < n_pos, with freq_i = 1.0f / powf(base, 2.0f*i/d_rot) and
 * angle = p * freq_i in float (src/ops/kernels.cpp:71-79). */
int mf_rope_table(float* out, int n_pos, int d_rot, float base);

/* y[0:d_out) = W · rmsnorm(x, norm_w, eps)  (rmsnorm + linear_proj,
 * module.cpp:187-191 fused; Q/K/V are one concatenated weight). */
int mf_rmsnorm_matmul(float* y, const float* x, const float* norm_w, float eps, const void* w, int dtype,
                      int d_out, int d_in, void* stream);

/* x[0:d_out) += W · a  (linear_proj + resadd, module.cpp:236-240). */
int mf_matmul_residual(float* x, const float* a, const void* w, int dtype, int d_out, int d_in, void* stream);

/* h[i] = silu(g_i) * u_i, g/u = rows 2i / 2i+1 of the interleaved gate/up
 * weight [2*d_ff, d_in] applied to rmsnorm(x)  (module.cpp:446,464-468). */
int mf_swiglu_matmul(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up, int dtype,
                     int d_ff, int d_in, void* stream);

/* Attention for one token (module.cpp:193-234 fused): per-head Q/K RMSNorm,
 * NeoX RoPE, append of K/V row `pos`, GQA attention over positions [0, pos].
 * qkv = [Hq*D | Hkv*D | Hkv*D] (output of the fused projection); caches are
 * [n_kv_heads][max_seq][d_head] fp32 for this layer. The workspace must hold
 * mf_attn_workspace_bytes() bytes and be zero-filled before its first use;
 * every call leaves its counters zero again. d_head must be 128. */
typedef struct mf_attn_desc {
    const float* qkv;
    const float* q_norm_w;
    const float* k_norm_w;
    float eps;
    const void* rope_table; /* mf_rope_table for >= max_seq positions (device) */
    void* k_cache;         /* this layer's [Hkv][max_seq][D] rows of kv_dtype */
    void* v_cache;
    int max_seq;
    const void* step_state; /* device step record (pos) */
    float* out;            /* [Hq*D] */
    int n_heads;
    int n_kv_heads;
    int d_head;
    int n_split;           /* position slices per KV head (mf_attn_default_split) */
    void* workspace;
    int kv_dtype;          /* MF_F32 (the reference's cache; 0, the default) or MF_BF16
                              (opt-in: rows rounded to nearest even at the append) */
} mf_attn_desc;
size_t mf_attn_workspace_bytes(int n_heads, int n_kv_heads, int d_head, int n_split);
int mf_attn_default_split(int n_kv_heads, int max_seq);
int mf_attn_decode(const mf_attn_desc* desc, void* stream);

/* Decode attention for callers that cannot allocate device memory (no
 * counterpart in the reference). Same computation and descriptor as
 * mf_attn_decode, but desc->workspace is ignored: the scratch is a static
 * device array of MF_ATTN_NOALLOC_SCRATCH_BYTES that every GPU loading this
 * library keeps until exit. For code that must not call cudaMalloc, e.g.
 * while a stream is captured in global mode, inside stream callbacks, or
 * when another runtime owns the device memory. The first call on a device
 * caches the array's address (make it before any stream capture); calls that
 * overlap on the GPU race on the shared array; a request needing more scratch
 * than the array holds returns MF_E_UNSUPPORTED. Allocates nothing. */
#define MF_ATTN_NOALLOC_SCRATCH_BYTES (1u << 20)
int mf_attn_decode_noalloc(const mf_attn_desc* desc, void* stream);

/* MoE router + top-k + renormalisation (module.cpp:446-457, kernels.cpp:113-139):
 * scores = W_router(f32 [E, d]) · rmsnorm(x); ids/weights of the k best. */
int mf_router_topk(int* ids, float* weights, float* scores, const float* x, const float* norm_w, float eps,
                   const float* w_router, int d_model, int n_experts, int k, void* stream);

/* Selected experts' SwiGLU (module.cpp:459-468): h[s*d_ff + i] for slot s < k
 * from the interleaved per-expert gate/up weight [E][2*d_ff][d_in]. */
int mf_moe_swiglu(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up_exps, int dtype,
                  const int* ids, int k, int d_ff, int d_in, void* stream);

/* Selected experts' down projection + weighted residual (module.cpp:469-474):
 * x[j] += sum over slots s in order of w_s * (W_down[ids[s]] · h_s)[j]. */
int mf_moe_down_residual(float* x, const float* h, const void* w_down_exps, int dtype, const int* ids,
                         const float* weights, int k, int d_model, int d_ff, void* stream);
/* The whole MoE FFN of one token (module.cpp:440-476): router + top-k
 * (scores, ids, weights: scratch outputs [n_experts], [k], [k]), the selected
 * experts' SwiGLU into h [k][d_ff], and the weighted down projection added to
 * x. Same results as the three calls above; launched as one chain, the down
 * projection's weight copies start while the gate/up kernel still runs. */
int mf_moe_ffn(float* x, float* h, const float* norm_w, float eps, const float* w_router, const void* w_gate_up_exps,
               const void* w_down_exps, int dtype, float* scores, int* ids, float* weights, int d_model, int d_ff,
               int n_experts, int k, void* stream);

/* Final RMSNorm + lm_head (module.cpp:54-79,113-126): logits = W · rmsnorm(x).
 * When step_state (a device step record) is non-NULL the greedy id (first
 * maximum, sampler.cpp:37) is written to its next_token field, and if its
 * chain field is non-zero the record advances (token = next_token, pos += 1)
 * for the next frame. The workspace (mf_lm_head_workspace_bytes, zero-filled
 * before first use) is then required. vocab_offset shifts the reported id
 * (vocab-split lm_head). */
size_t mf_lm_head_workspace_bytes(void);
int mf_lm_head(float* logits, const float* x, const float* norm_w, float eps, const void* w, int dtype, int vocab,
               int d_model, int vocab_offset, void* step_state, void* workspace, void* stream);

/* ===================================================================== */
/* Tensor parallelism over NVLink / NVSwitch peer memory                 */
/* ===================================================================== */
/* No reference counterpart: the reference runs one device
 * (src/base/model.cpp:36-59). These calls split each decoder layer over
 * tp_size GPUs, one process per GPU: Q/K/V by KV-head group, O by input
 * columns, gate/up by FFN rows, down by FFN columns, lm_head by vocabulary
 * rows; embeddings and norms are replicated. The two all-reduces per layer
 * are fused into the GEMVs around them: the O and down projections store
 * their partial rows straight into every rank's receive slot
 * (mf_matmul_push), and the next RMSNorm GEMV reads all ranks' partials in
 * its prologue and sums them in rank order with the residual
 * (mf_allreduce_*). Each value travels in one 64-bit store with a 32-bit tag
 * (frame * 256 + seq, frame from the step record's MF_STEP_FRAME field), so
 * no memory fence or flag round trip is needed; waits are bounded by
 * MF_COMM_TIMEOUT_MS (default 1000) and a wait that gives up sets a bit
 * readable with mf_comm_status. No TMA, no multicast.
 *
 * Setup: mf_comm_create on every rank, exchange the MF_COMM_HANDLE_BYTES
 * handles (any host channel, e.g. torch.distributed), mf_comm_connect with
 * all handles ordered by tp_rank. Every rank then issues the same sequence of
 * frames and exchange calls. `seq` numbers the exchanges within one frame
 * (0 .. 254; consecutive exchanges alternate its parity, e.g. 2*layer and
 * 2*layer + 1), and the step record's frame field must advance between
 * frames. */
#define MF_TP_MAX 8
#define MF_COMM_HANDLE_BYTES 64
typedef struct mf_comm mf_comm;
/* max_floats: longest all-reduced vector (d_model, multiple of 4);
 * gather_floats: length of the full-logits gather buffer (vocabulary size, or 0). */
int mf_comm_create(int rank, int tp_rank, int tp_size, int max_floats, int gather_floats, mf_comm** out);
/* The same with two bulk slots of bulk_floats fp32 each for batched-prefill
 * exchanges of [rows, d] partials (mf_comm_bulk_ptr, mf_bulk_allreduce). */
int mf_comm_create_ex(int rank, int tp_rank, int tp_size, int max_floats, int gather_floats, size_t bulk_floats,
                      mf_comm** out);
int mf_comm_handle(const mf_comm* c, void* out, size_t n);
/* A rank's own handle in another rank's place maps that peer to this rank's
 * region: a loopback in which that peer never sends (its waits time out). */
int mf_comm_connect(mf_comm* c, const void* handles, size_t n);
/* COMM status bits (1: an all-reduce wait gave up, 2: a greedy-id exchange
 * gave up); clear != 0 resets them. Synchronises the rank's stream. */
int mf_comm_status(mf_comm* c, int* status, int clear);
/* Device address of this rank's full-logits buffer (mf_allreduce_lm_head with gather_logits). */
int mf_comm_gather_ptr(const mf_comm* c, float** logits);
/* This rank's bulk slot (0 or 1): where its partial of a batched-prefill
 * exchange goes (for example as the output of mf_prefill_gemm). */
int mf_comm_bulk_ptr(const mf_comm* c, int slot, float** out);
/* Batched-prefill all-reduce (replaces minfer's per-token exchange-free CPU
 * path, src/base/model.cpp:120-129, for tensor-parallel shards): after this
 * rank's partial is complete in bulk slot `slot`, x[i] += (partial_0[i] + ...
 * + partial_{T-1}[i]) with the sum in rank order, the same on every rank
 * (reduce-scatter into the slots, then all-gather; the slot's contents are
 * consumed). `epoch` numbers the
 * exchanges (1, 2, ... identical on every rank); slots must alternate between
 * consecutive exchanges. A wait that gives up sets mf_comm_status bit 1 and
 * leaves x unchanged. */
int mf_bulk_allreduce(float* x, size_t n, mf_comm* c, int slot, unsigned long long epoch, void* stream);
void mf_comm_destroy(mf_comm* c);

/* All-reduce send fused into a GEMV: the partial W·a of this rank (W holds
 * this rank's input columns) goes to every rank as exchange `seq`. */
int mf_matmul_push(const float* a, const void* w, int dtype, int d_out, int d_in, mf_comm* c, int seq,
                   const void* step_state, void* stream);
/* All-reduce receive fused into an RMSNorm GEMV: x = x_res + sum of every
 * rank's partial of exchange `seq` (rank order), x_out = x (written once),
 * y = W · rmsnorm(x) (W holds this rank's output rows). */
int mf_allreduce_rmsnorm_matmul(float* y, const float* x_res, float* x_out, const float* norm_w, float eps,
                                const void* w, int dtype, int d_out, int d_in, mf_comm* c, int seq,
                                const void* step_state, void* stream);
/* The same receive fused into the SwiGLU gate/up GEMV (d_ff = this rank's rows). */
int mf_allreduce_swiglu_matmul(float* h, const float* x_res, float* x_out, const float* norm_w, float eps,
                               const void* w_gate_up, int dtype, int d_ff, int d_in, mf_comm* c, int seq,
                               const void* step_state, void* stream);
/* The same receive fused into the vocabulary-split lm_head: logits rows
 * [vocab_offset, vocab_offset + vocab) of this rank. The greedy id is agreed
 * over all ranks (every rank writes the same id to its step record and, for
 * a chained record, advances it); with gather_logits every rank also receives
 * all ranks' logits in its gather buffer (mf_comm_gather_ptr), complete when
 * the kernel ends. step_state and workspace are required. */
int mf_allreduce_lm_head(float* logits, const float* x_res, float* x_out, const float* norm_w, float eps,
                         const void* w, int dtype, int vocab, int d_model, int vocab_offset, void* step_state,
                         void* workspace, int gather_logits, mf_comm* c, int seq, void* stream);
/* Tensor-parallel MoE layer (no reference counterpart): receive the
 * attention all-reduce (exchange seq) into x_out (as mf_allreduce_rmsnorm_matmul),
 * then the router GEMV over rmsnorm(x_out) and the top-k as mf_router_topk.
 * The experts then run on this rank's slice of their FFN rows
 * (mf_moe_swiglu on x_out, then mf_moe_down_push with every expert local). */
int mf_allreduce_router_topk(int* ids, float* weights, float* scores, const float* x_res, float* x_out,
                             const float* norm_w, float eps, const float* w_router, int d_model, int n_experts, int k,
                             mf_comm* c, int seq, const void* step_state, void* stream);
/* Expert parallelism (MoE): each rank stores experts [expert_lo,
 * expert_lo + n_local) (expert e at local index e - expert_lo); the router
 * runs on every rank, so all ranks hold the same ids. h of slots routed to
 * another rank's experts is left undefined here (the down projection skips
 * those slots). mf_moe_swiglu_ep is mf_moe_swiglu over
 * the local experts; mf_moe_down_push computes this rank's weighted sum of its
 * experts' down projections (slot order) and sends it as exchange `seq`, to be
 * received by the next mf_allreduce_* call (the residual add happens there). */
int mf_moe_swiglu_ep(float* h, const float* x, const float* norm_w, float eps, const void* w_gate_up_local, int dtype,
                     const int* ids, int k, int d_ff, int d_in, int expert_lo, int n_local, void* stream);
int mf_moe_down_push(const float* h, const void* w_down_local, int dtype, const int* ids, const float* weights, int k,
                     int d_model, int d_ff, int expert_lo, int n_local, mf_comm* c, int seq, const void* step_state,
                     void* stream);
/* Stand-alone all-reduce of n floats (one kernel): x_out = x_res + sum over
 * ranks of `partial` (rank order). x_out may equal x_res. */
int mf_allreduce(float* x_out, const float* x_res, const float* partial, int n, mf_comm* c, int seq,
                 const void* step_state, void* stream);

/* ===================================================================== */
/* Batched prefill (tcgen05 tensor cores)                                */
/* ===================================================================== */
/* No reference counterpart: the reference prefills token by token
 * (src/base/model.cpp:120-129). These calls process all n_tokens prompt
 * tokens of a layer at once. Activations stay fp32 between calls; a GEMM
 * operand is the fp32 activation split into two bf16 matrices hi + lo
 * (hi = bf16(a), lo = bf16(a - hi)), so bf16 tensor cores reproduce the
 * fp32-activation GEMV to ~1e-5 relative. bf16 matrices are row-major,
 * 16-byte aligned, row length a multiple of 8. */
#define MF_PREFILL_STORE 0  /* y[m*ldy + n] = C */
#define MF_PREFILL_RESID 1  /* y[m*ldy + n] += C */
#define MF_PREFILL_SWIGLU 2 /* C's columns 2i/2i+1 are gate_i/up_i: h = silu(g)*u as hi/lo [M][N/2] */
/* C[M, N] = (a_hi + a_lo)[M, K] · w[N, K]^T with w bf16. */
int mf_prefill_gemm(float* y, int ldy, const void* a_hi, const void* a_lo, const void* w, int M, int N, int K,
                    int mode, void* h_hi, void* h_lo, void* stream);
/* Grouped form (MoE experts): n_groups problems C_g = A_g · w_g^T, where A_g
 * is rows [grp_rows[g], grp_rows[g+1]) of a_hi/a_lo [rows_cap][K], w_g the
 * g-th [N][K] matrix of w, and group g's 128-row tiles are numbered from
 * grp_tiles[g] (grp_rows / grp_tiles: device arrays of n_groups + 1 entries,
 * e.g. from mf_prefill_moe_group). C rows keep A's row numbers. */
int mf_prefill_gemm_grouped(float* y, int ldy, const void* a_hi, const void* a_lo, const void* w, int n_groups,
                            int rows_cap, int N, int K, const int* grp_rows, const int* grp_tiles, int mode,
                            void* h_hi, void* h_lo, void* stream);
/* MoE layer prefill pieces (src/models/qwen3/module.cpp:440-476 for n tokens):
 * route: fp32 router scores of the normalised rows xn [n_tokens][d_model]
 *   against w_router [n_experts][d_model] and the reference's top-k + softmax
 *   per token -> ids / weights [n_tokens][k] (n_experts a multiple of 4, <= 256);
 * group: counting sort of the n_tokens*k (token, slot) pairs by expert, over
 *   the experts [expert_lo, expert_lo + n_local) stored here: rows / tiles
 *   [n_local + 1] (first grouped row / 128-row tile of each local expert) and
 *   pos [n_tokens*k] (the grouped row of pair t*k + s, -1 for an expert
 *   stored elsewhere);
 * gather: token t's row of xn split into bf16 hi/lo at its grouped rows;
 * combine: x_out[t] = x_in[t] (0 when x_in is null) + weights[t][s] *
 *   y[pos[t*k + s]] for s = 0..k-1 in order, slots with pos -1 skipped. */
int mf_prefill_moe_route(int* ids, float* weights, const float* xn, const float* w_router, int n_tokens, int d_model,
                         int n_experts, int k, void* stream);
int mf_prefill_moe_group(const int* ids, int n_tokens, int k, int expert_lo, int n_local, int* rows, int* tiles,
                         int* pos, void* stream);
int mf_prefill_moe_gather(void* a_hi, void* a_lo, const float* xn, const int* pos, int n_tokens, int k, int d_model,
                          void* stream);
int mf_prefill_moe_combine(float* x_out, const float* x_in, const float* y, const int* pos, const float* weights,
                           int n_tokens, int k, int d_model, void* stream);
/* Row-wise RMSNorm (src/ops/kernels.cpp:351-365) of x [n_rows][d] split into
 * bf16 hi/lo; xn (optional) receives the fp32 normalised rows. */
int mf_prefill_norm_split(void* hi, void* lo, float* xn, const float* x, const float* norm_w, float eps, int d,
                          int n_rows, void* stream);
/* fp32 -> bf16 hi/lo split of n elements. */
int mf_prefill_split(void* hi, void* lo, const float* x, size_t n, void* stream);
/* h = silu(g) * u (src/models/qwen3/module.cpp:466-468) of fp32 gate/up rows
 * [n_rows][2 d_ff] (columns 2i, 2i+1 = g_i, u_i), as bf16 hi/lo [n_rows][d_ff]:
 * the SwiGLU step of fp32-weight models, whose gate/up GEMM runs as two
 * products (weights split into bf16 hi + lo) that are summed before it. */
int mf_prefill_swiglu_split(void* h_hi, void* h_lo, const float* gate_up, int n_rows, int d_ff, void* stream);
/* x[t] = embedding row tokens[t] (device ids) for t < n_tokens. */
int mf_prefill_embed(float* x, const void* emb, int dtype, int vocab, int d_model, const uint32_t* tokens,
                     int n_tokens, void* stream);
/* Per token t (position pos0 + t) of qkv [n_tokens][(Hq + 2 Hkv) * d_head]:
 * Q/K RMSNorm + NeoX RoPE (as mf_attn_decode), q -> q_out [n_tokens][Hq * d_head],
 * k/v -> cache row pos0 + t (caches [n_kv_heads][max_seq][d_head] of kv_dtype,
 * MF_F32 or MF_BF16, this layer). */
int mf_prefill_qkv_post(float* q_out, void* k_cache, void* v_cache, const float* qkv, const float* q_norm_w,
                        const float* k_norm_w, float eps, const void* rope_table, int max_seq, int n_heads,
                        int n_kv_heads, int d_head, int n_tokens, int pos0, int kv_dtype, void* stream);
/* Causal GQA attention of the prompt tokens (token t sees cache rows
 * [0, pos0 + t]), written as bf16 hi/lo [n_tokens][Hq * d_head]. */
int mf_prefill_attention(void* out_hi, void* out_lo, const float* q, const void* k_cache, const void* v_cache,
                         int max_seq, int n_tokens, int pos0, int n_heads, int n_kv_heads, int d_head, int kv_dtype,
                         void* stream);
/* The same attention on the tensor cores (tcgen05): S = Q K^T with fp16 hi/lo
 * operands and O += P V with bf16 hi/lo operands (three products each) in
 * TMEM, online softmax per query row. Needs device scratch of at least
 * mf_prefill_attention_scratch(n_tokens, pos0 + n_tokens, ...) bytes,
 * 256-byte aligned. A wait that gives up sets status bit 2; a q or k value
 * outside the fp16 range (|x| >= 65504, or not finite) sets status bit 4. */
int mf_prefill_attention_scratch(int n_tokens, int n_keys, int n_heads, int n_kv_heads, size_t* bytes);
int mf_prefill_attention_tc(void* out_hi, void* out_lo, const float* q, const void* k_cache, const void* v_cache,
                            int max_seq, int n_tokens, int pos0, int n_heads, int n_kv_heads, int d_head,
                            void* scratch, size_t scratch_bytes, int kv_dtype, void* stream);
/* ===================================================================== */
/* Sampling on the device                                                */
/* ===================================================================== */
/* The k (<= 64) largest of x[0, n) and their indices, sorted by value,
 * largest first (equal values: lower index first; NaN counts as -inf): the
 * candidate list minfer's Sampler builds with nth_element + sort
 * (src/base/sampler.cpp:40-50), so the host only needs k pairs instead of the
 * whole vocabulary. The workspace (mf_topk_workspace_bytes, 16-byte aligned)
 * must be zero before the first call; the kernel leaves it ready for the next. */
size_t mf_topk_workspace_bytes(int n, int k);
int mf_topk(const float* x, int n, int k, int* ids, float* vals, void* workspace, size_t workspace_bytes,
            void* stream);
/* One sampled token on the device from a top-k candidate list (top_k + 1
 * entries from mf_topk, so equal logits at the cut are seen): the reference's
 * Sampler::sample after its top-k (softmax, top-p, min-p, temperature softmax,
 * the first candidate whose cumulative probability reaches draws[i], i = the
 * step record's MF_STEP_SAMPLE field). The chosen id is written to out_ids[i]
 * and becomes the record's token; position, frame and sample index advance,
 * so a captured frame can feed the next one. flags: bit 1 equal logits among
 * the candidates, bit 2 sample index outside [0, n_draws), bit 4 every
 * candidate filtered out. No presence penalty (it changes the list). */
int mf_sample_step(const int* cand_ids, const float* cand_vals, int top_k, float temp, float top_p, float min_p,
                   const float* draws, int n_draws, void* step_state, int* out_ids, int* flags, void* stream);

/* Status bits of the prefill kernels since the last clear (1: a GEMM wait
 * gave up, 2: an attention wait gave up, 4: attention q/k outside the fp16
 * range; synchronises the device). */
int mf_prefill_status(int* status, int clear);

/* ===================================================================== */
/* Single ops with the reference's CPU signatures                        */
/* (include/minfer/ops/kernels.hpp:13-32) on device buffers.              */
/* ===================================================================== */
int mf_matmul(float* y, const float* x, const void* w, int dtype, size_t offset, int d_out, int d_in, void* stream);
int mf_rmsnorm(float* out, const float* x, const float* w, int dim, float eps, int n_rows, void* stream);
int mf_softmax(float* out, const float* x, int n, int n_rows, void* stream);
int mf_silu(float* out, const float* x, int n, void* stream);
int mf_neox_rope(float* out, const float* x, int head, int d_head, int d_rot, float base, int pos, void* stream);
int mf_il_rope(float* out, const float* x, int head, int d_head, int d_rot, float base, int pos, void* stream);
int mf_attn(float* scores, float* out, const float* q, const float* k, const float* v, int seq_len, int d_head,
            int kv_dim, void* stream);
int mf_route(const float* x, int* ids, float* weights, float* scores, const float* w_router, int d_model,
             int n_experts, int k, void* stream);
int mf_embed(float* x, const void* w, int dtype, uint32_t token, int d_model, void* stream);
int mf_argmax(const float* logits, int n, int* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MINFER_CUDA_H */
