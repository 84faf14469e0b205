#include "model.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <random>
#include <stdexcept>

namespace minfer {

namespace {

void check(int rc, const char* what) {
    if (rc != MF_OK) {
        char msg[512];
        mf_last_error(msg, sizeof(msg));
        throw std::runtime_error(std::string(what) + " failed (" + std::to_string(rc) + "): " + msg);
    }
}

int mf_dtype(DataType t) {
    switch (t) {
        case DataType::F32: return MF_F32;
        case DataType::F16: return MF_F16;
        case DataType::BF16: return MF_BF16;
        default: throw std::runtime_error("unsupported weight dtype");
    }
}

// Tensor-parallel batched prefill: a projection's partial goes into this
// rank's next bulk slot (exchange rs.pf_epoch + 1, slots alternating), then
// X += every rank's partial in rank order.
float* prefill_exchange_slot(RunState& rs) {
    float* p = nullptr;
    check(mf_comm_bulk_ptr(rs.comm, (int)((rs.pf_epoch + 1) & 1), &p), "prefill exchange slot");
    return p;
}
void prefill_exchange(RunState& rs, float* X, int n, int d) {
    const unsigned long long ep = ++rs.pf_epoch;
    check(mf_bulk_allreduce(X, (size_t)n * d, rs.comm, (int)(ep & 1), ep, rs.stream), "prefill all-reduce");
}

// fp32 weights for the batched prefill: the tensor-core GEMM takes bf16
// weights, so an fp32 matrix is kept as bf16 hi + lo (w = hi + lo to ~2^-17
// relative) and multiplied as two products summed in fp32.
struct SplitWeight {
    mf_buf *hi = nullptr, *lo = nullptr;
};
SplitWeight split_weight(mf_buf* w, size_t n, int rank) {
    SplitWeight s;
    check(mf_alloc(n * 2, rank, &s.hi), "alloc weight hi");
    check(mf_alloc(n * 2, rank, &s.lo), "alloc weight lo");
    check(mf_prefill_split(mf_ptr(s.hi), mf_ptr(s.lo), (const float*)mf_ptr(w), n, mf_stream(rank)), "split weight");
    check(mf_sync(rank), "sync");
    return s;
}

// C = A · W^T for a prefill GEMM in `mode`, W bf16 or (fp32 models) a split
// pair: the hi product in `mode`, then the lo product added (MF_PREFILL_RESID).
void prefill_gemm(float* y, int ldy, void* a_hi, void* a_lo, const mf_buf* w, const SplitWeight& sw, int M, int N,
                  int K, int mode, void* stream, const char* what) {
    if (!sw.hi) {
        check(mf_prefill_gemm(y, ldy, a_hi, a_lo, mf_ptr(w), M, N, K, mode, nullptr, nullptr, stream), what);
        return;
    }
    check(mf_prefill_gemm(y, ldy, a_hi, a_lo, mf_ptr(sw.hi), M, N, K, mode, nullptr, nullptr, stream), what);
    check(mf_prefill_gemm(y, ldy, a_hi, a_lo, mf_ptr(sw.lo), M, N, K, MF_PREFILL_RESID, nullptr, nullptr, stream),
          what);
}

mf_buf* upload_tensor(const TensorView& t, int rank) {
    mf_buf* b = nullptr;
    check(mf_upload(t.data, t.bytes, rank, &b), ("upload " + t.name).c_str());
    return b;
}

void expect_shape(const TensorView& t, std::initializer_list<uint64_t> shape) {
    std::vector<uint64_t> want(shape);
    if (t.shape != want) {
        std::string w, g;
        for (auto v : want) w += std::to_string(v) + " ";
        for (auto v : t.shape) g += std::to_string(v) + " ";
        throw std::runtime_error("tensor " + t.name + " has shape [" + g + "], expected [" + w + "]");
    }
}

// Rows [r0, r0 + n) of a row-major tensor, uploaded as one contiguous buffer.
mf_buf* upload_rows(const TensorView& t, size_t r0, size_t n, size_t row_bytes, int rank) {
    if ((r0 + n) * row_bytes > t.bytes) throw std::runtime_error("row slice outside tensor " + t.name);
    mf_buf* b = nullptr;
    check(mf_upload((const char*)t.data + r0 * row_bytes, n * row_bytes, rank, &b), ("upload " + t.name).c_str());
    return b;
}

// Columns [c0, c0 + nc) (in bytes: col0_bytes, width_bytes) of every row of a
// row-major [rows, row_bytes] tensor, packed into a new [rows, width] buffer.
mf_buf* upload_cols(const TensorView& t, size_t rows, size_t row_bytes, size_t col0_bytes, size_t width_bytes,
                    int rank) {
    if (rows * row_bytes != t.bytes || col0_bytes + width_bytes > row_bytes)
        throw std::runtime_error("column slice outside tensor " + t.name);
    mf_buf* b = nullptr;
    check(mf_alloc(rows * width_bytes, rank, &b), ("alloc " + t.name).c_str());
    check(mf_write_2d(b, 0, width_bytes, (const char*)t.data + col0_bytes, row_bytes, width_bytes, rows),
          ("upload " + t.name).c_str());
    return b;
}

void expect_f32(const TensorView& t) {
    // norms and the router are fp32 (src/base/module.cpp:64,88-93,130-134)
    if (t.dtype != DataType::F32) throw std::runtime_error("tensor " + t.name + " must be F32");
}

double now_s() {
    using namespace std::chrono;
    return duration_cast<duration<double>>(steady_clock::now().time_since_epoch()).count();
}

// ---------------------------------------------------------------- layers

// Qwen3Embed (src/models/qwen3/module.cpp:13-44)
class Qwen3Embed : public BaseLayer {
public:
    Qwen3Embed(const Config& c) : c_(c) {}
    void upload(const GGUFFile& f, int rank) override {
        const TensorView& t = f.tensor("token_embd.weight");
        expect_shape(t, {c_.vocab_size, (uint64_t)c_.d_model});
        dtype_ = mf_dtype(t.dtype);
        w_ = upload_tensor(t, rank);
        own(w_);
        read_bytes_ = t.bytes / c_.vocab_size;  // one row (src/base/module.cpp:33)
    }
    void cuda_forward(RunState& rs) override {
        check(mf_embed_step((float*)mf_ptr(rs.x), mf_ptr(w_), dtype_, (int)c_.vocab_size, c_.d_model, rs.d_step,
                            rs.stream),
              "embed");
    }
    void prefill_forward(RunState& rs, int n, int pos0) override {
        check(mf_prefill_embed((float*)mf_ptr(rs.pf_x), mf_ptr(w_), dtype_, (int)c_.vocab_size, c_.d_model,
                               (const uint32_t*)mf_ptr(rs.pf_tok), n, rs.stream),
              "prefill embed");
    }
    mf_buf* weight() const { return w_; }
    int dtype() const { return dtype_; }

private:
    const Config& c_;
    mf_buf* w_ = nullptr;
    int dtype_ = MF_F32;
};

// Qwen3GQA (src/models/qwen3/module.cpp:142-241)
class Qwen3GQA : public BaseLayer {
public:
    Qwen3GQA(const Config& c, int layer) : c_(c), layer_(layer) {}
    void upload(const GGUFFile& f, int rank) override {
        const std::string p = "blk." + std::to_string(layer_) + ".";
        const TensorView& wq = f.tensor(p + "attn_q.weight");
        const TensorView& wk = f.tensor(p + "attn_k.weight");
        const TensorView& wv = f.tensor(p + "attn_v.weight");
        const TensorView& wo = f.tensor(p + "attn_output.weight");
        const TensorView& qn = f.tensor(p + "attn_q_norm.weight");
        const TensorView& kn = f.tensor(p + "attn_k_norm.weight");
        const TensorView& an = f.tensor(p + "attn_norm.weight");
        const uint64_t d = c_.d_model, q = (uint64_t)c_.n_heads * c_.d_head, kv = (uint64_t)c_.n_kv_heads * c_.d_head;
        expect_shape(wq, {q, d});
        expect_shape(wk, {kv, d});
        expect_shape(wv, {kv, d});
        expect_shape(wo, {d, q});
        expect_shape(qn, {(uint64_t)c_.d_head});
        expect_shape(kn, {(uint64_t)c_.d_head});
        expect_shape(an, {d});
        if (!(wq.dtype == wk.dtype && wk.dtype == wv.dtype && wv.dtype == wo.dtype))
            throw std::runtime_error("Q/K/V/O weights of layer " + std::to_string(layer_) + " differ in dtype");
        expect_f32(qn);
        expect_f32(kn);
        expect_f32(an);
        dtype_ = mf_dtype(wq.dtype);
        // fused [Wq; Wk; Wv] so one streaming pass computes q|k|v; under
        // tensor parallelism this rank's KV-head group: Q heads and K/V heads
        // [t*H/T, (t+1)*H/T), and the matching input columns of Wo
        const size_t esz = dtype_size(wq.dtype), rowb = d * esz, t = c_.attn_split() ? c_.tp_rank : 0;
        const size_t ql = (size_t)c_.heads_local() * c_.d_head, kvl = (size_t)c_.kv_heads_local() * c_.d_head;
        const char* qsrc = (const char*)wq.data + t * ql * rowb;
        const char* ksrc = (const char*)wk.data + t * kvl * rowb;
        const char* vsrc = (const char*)wv.data + t * kvl * rowb;
        check(mf_alloc((ql + 2 * kvl) * rowb, rank, &wqkv_), "alloc qkv");
        check(mf_write(wqkv_, 0, qsrc, ql * rowb), "upload q");
        check(mf_write(wqkv_, ql * rowb, ksrc, kvl * rowb), "upload k");
        check(mf_write(wqkv_, (ql + kvl) * rowb, vsrc, kvl * rowb), "upload v");
        own(wqkv_);
        own(wo_ = !c_.attn_split() ? upload_tensor(wo, rank) : upload_cols(wo, d, q * esz, t * ql * esz, ql * esz, rank));
        own(qn_ = upload_tensor(qn, rank));
        own(kn_ = upload_tensor(kn, rank));
        own(an_ = upload_tensor(an, rank));
        // normalised, rotated q/k elements are bounded by sqrt(2 * d_head) * max|norm weight|; the
        // tensor-core prefill attention carries them as fp16 hi/lo, so it needs that bound below 65504
        float wmax = 0.f;
        for (const TensorView* tv : {&qn, &kn})
            for (size_t i = 0; i < tv->numel; ++i) wmax = std::max(wmax, std::fabs(((const float*)tv->data)[i]));
        tc_attn_ok_ = std::sqrt(2.0f * (float)c_.d_head) * wmax < 60000.f;
        read_bytes_ = (ql + 2 * kvl) * rowb + d * ql * esz + qn.bytes + kn.bytes + an.bytes;
        if (c_.ep()) read_bytes_ /= c_.tp_size;  // replicated: each rank counts its share
    }
    void cuda_forward(RunState& rs) override {
        const int d = c_.d_model, H = c_.heads_local(), Hkv = c_.kv_heads_local(), D = c_.d_head;
        // expert parallelism: the residual of layer l lives in xb[l & 1]; the
        // previous layer's expert all-reduce (exchange l - 1) is received here
        float* xres = c_.ep() ? (float*)mf_ptr(rs.xb[layer_ & 1]) : (float*)mf_ptr(rs.x);
        if (c_.tp_size == 1 || layer_ == 0) {
            check(mf_rmsnorm_matmul((float*)mf_ptr(rs.qkv), (const float*)mf_ptr(rs.x), (const float*)mf_ptr(an_),
                                    c_.rms_norm_eps, mf_ptr(wqkv_), dtype_, (H + 2 * Hkv) * D, d, rs.stream),
                  "qkv projection");
        } else if (c_.ep()) {
            check(mf_allreduce_rmsnorm_matmul((float*)mf_ptr(rs.qkv), (const float*)mf_ptr(rs.xb[(layer_ - 1) & 1]),
                                              xres, (const float*)mf_ptr(an_), c_.rms_norm_eps, mf_ptr(wqkv_), dtype_,
                                              (H + 2 * Hkv) * D, d, rs.comm, layer_ - 1, rs.d_step, rs.stream),
                  "qkv projection (expert all-reduce)");
        } else {
            // receive the previous layer's down-projection all-reduce
            check(mf_allreduce_rmsnorm_matmul((float*)mf_ptr(rs.qkv), (const float*)mf_ptr(rs.xb[1]),
                                              (float*)mf_ptr(rs.xb[0]), (const float*)mf_ptr(an_), c_.rms_norm_eps,
                                              mf_ptr(wqkv_), dtype_, (H + 2 * Hkv) * D, d, rs.comm, 2 * layer_ - 1,
                                              rs.d_step, rs.stream),
                  "qkv projection (all-reduce)");
        }
        mf_attn_desc a = {};
        a.qkv = (const float*)mf_ptr(rs.qkv);
        a.q_norm_w = (const float*)mf_ptr(qn_);
        a.k_norm_w = (const float*)mf_ptr(kn_);
        a.eps = c_.rms_norm_eps;
        a.rope_table = mf_ptr(rs.rope);
        a.k_cache = rs.kv_layer(rs.k_cache, layer_);
        a.v_cache = rs.kv_layer(rs.v_cache, layer_);
        a.kv_dtype = rs.kv_dtype;
        a.max_seq = (int)c_.user_max_seq_len;
        a.step_state = rs.d_step;
        a.out = (float*)mf_ptr(rs.att);
        a.n_heads = H;
        a.n_kv_heads = Hkv;
        a.d_head = D;
        a.n_split = rs.attn_split;
        a.workspace = mf_ptr(rs.attn_ws);
        check(mf_attn_decode(&a, rs.stream), "attention");
        if (!c_.attn_split()) {
            check(mf_matmul_residual(xres, (const float*)mf_ptr(rs.att), mf_ptr(wo_), dtype_, d, H * D, rs.stream),
                  "output projection");
        } else {
            check(mf_matmul_push((const float*)mf_ptr(rs.att), mf_ptr(wo_), dtype_, d, H * D, rs.comm, 2 * layer_,
                                 rs.d_step, rs.stream),
                  "output projection (all-reduce send)");
        }
    }

    // the same layer for n prompt tokens at once: pre-norm, QKV GEMM, Q/K norm
    // + RoPE + KV write, causal attention, O GEMM + residual
    void prefill_forward(RunState& rs, int n, int pos0) override {
        const int d = c_.d_model, H = c_.heads_local(), Hkv = c_.kv_heads_local(), D = c_.d_head;
        const int Nqkv = (H + 2 * Hkv) * D;
        const int S = (int)c_.user_max_seq_len;
        float* X = (float*)mf_ptr(rs.pf_x);
        void *hi = mf_ptr(rs.pf_hi), *lo = mf_ptr(rs.pf_lo);
        void* kc = rs.kv_layer(rs.k_cache, layer_);
        void* vc = rs.kv_layer(rs.v_cache, layer_);
        check(mf_prefill_norm_split(hi, lo, nullptr, X, (const float*)mf_ptr(an_), c_.rms_norm_eps, d, n, rs.stream),
              "prefill attn norm");
        prefill_gemm((float*)mf_ptr(rs.pf_qkv), Nqkv, hi, lo, wqkv_, wqkv_s_, n, Nqkv, d, MF_PREFILL_STORE, rs.stream,
                     "prefill qkv projection");
        check(mf_prefill_qkv_post((float*)mf_ptr(rs.pf_q), kc, vc, (const float*)mf_ptr(rs.pf_qkv),
                                  (const float*)mf_ptr(qn_), (const float*)mf_ptr(kn_), c_.rms_norm_eps,
                                  mf_ptr(rs.rope), S, H, Hkv, D, n, pos0, rs.kv_dtype, rs.stream),
              "prefill q/k norm, rope, kv");
        if (rs.pf_simt_attn || !tc_attn_ok_)
            check(mf_prefill_attention(hi, lo, (const float*)mf_ptr(rs.pf_q), kc, vc, S, n, pos0, H, Hkv, D,
                                       rs.kv_dtype, rs.stream),
                  "prefill attention");
        else
            check(mf_prefill_attention_tc(hi, lo, (const float*)mf_ptr(rs.pf_q), kc, vc, S, n, pos0, H, Hkv, D,
                                          mf_ptr(rs.pf_att), rs.pf_att_bytes, rs.kv_dtype, rs.stream),
                  "prefill attention");
        if (!c_.attn_split()) {  // one GPU, or expert parallelism (attention replicated)
            prefill_gemm(X, d, hi, lo, wo_, wo_s_, n, d, H * D, MF_PREFILL_RESID, rs.stream,
                         "prefill output projection");
        } else {
            float* part = prefill_exchange_slot(rs);
            prefill_gemm(part, d, hi, lo, wo_, wo_s_, n, d, H * D, MF_PREFILL_STORE, rs.stream,
                         "prefill output projection (partial)");
            prefill_exchange(rs, X, n, d);
        }
    }
    // fp32 weights: bf16 hi/lo copies for the batched prefill (made on first use)
    void split_for_prefill(int rank) override {
        if (dtype_ != MF_F32 || wqkv_s_.hi) return;
        const size_t d = c_.d_model, ql = (size_t)c_.heads_local() * c_.d_head, kvl = (size_t)c_.kv_heads_local() * c_.d_head;
        wqkv_s_ = split_weight(wqkv_, (ql + 2 * kvl) * d, rank);
        wo_s_ = split_weight(wo_, d * ql, rank);
        for (mf_buf* b : {wqkv_s_.hi, wqkv_s_.lo, wo_s_.hi, wo_s_.lo}) own(b);
    }

private:
    const Config& c_;
    int layer_;
    int dtype_ = MF_BF16;
    mf_buf *wqkv_ = nullptr, *wo_ = nullptr, *qn_ = nullptr, *kn_ = nullptr, *an_ = nullptr;
    SplitWeight wqkv_s_, wo_s_;  // fp32 models: prefill copies
    bool tc_attn_ok_ = true;  // q/k fit the tensor-core attention's fp16 operands
};

// Qwen3MoE (src/models/qwen3/module.cpp:405-476): dense SwiGLU FFN when the
// model has no experts (the reference's "expert 0 with weight 1").
class Qwen3MoE : public BaseLayer {
public:
    Qwen3MoE(const Config& c, int layer) : c_(c), layer_(layer) {}
    void upload(const GGUFFile& f, int rank) override {
        const std::string p = "blk." + std::to_string(layer_) + ".";
        const bool moe = c_.n_experts > 0;
        const TensorView& fn = f.tensor(p + "ffn_norm.weight");
        const TensorView& wg = f.tensor(p + (moe ? "ffn_gate_exps.weight" : "ffn_gate.weight"));
        const TensorView& wu = f.tensor(p + (moe ? "ffn_up_exps.weight" : "ffn_up.weight"));
        const TensorView& wd = f.tensor(p + (moe ? "ffn_down_exps.weight" : "ffn_down.weight"));
        const uint64_t d = c_.d_model, F = c_.d_ff, E = c_.n_experts;
        expect_shape(fn, {d});
        expect_f32(fn);
        if (moe) {
            expect_shape(wg, {E, F, d});
            expect_shape(wu, {E, F, d});
            expect_shape(wd, {E, d, F});
        } else {
            expect_shape(wg, {F, d});
            expect_shape(wu, {F, d});
            expect_shape(wd, {d, F});
        }
        if (!(wg.dtype == wu.dtype && wu.dtype == wd.dtype))
            throw std::runtime_error("FFN weights of layer " + std::to_string(layer_) + " differ in dtype");
        dtype_ = mf_dtype(wg.dtype);
        own(fn_ = upload_tensor(fn, rank));
        // gate/up interleaved by row: row 2i = gate_i, 2i+1 = up_i (per expert);
        // under tensor parallelism (dense) this rank's FFN rows
        // [t*F/T, (t+1)*F/T) and the matching input columns of W_down
        const size_t esz = dtype_size(wg.dtype), row = (size_t)d * esz;
        const size_t Fl = (size_t)c_.ff_local(), t = c_.attn_split() ? c_.tp_rank : 0;
        if (moe && c_.moe_tp) {
            // every expert's FFN rows [t*Fl, (t+1)*Fl) (gate/up interleaved per
            // expert) and the matching input columns of its down matrix
            check(mf_alloc(2 * E * Fl * row, rank, &wgu_), "alloc gate/up");
            check(mf_alloc(E * d * Fl * esz, rank, &wd_), "alloc down");
            for (size_t e = 0; e < E; ++e) {
                const size_t src = (e * F + t * Fl) * row, dst = e * 2 * Fl * row;
                check(mf_write_2d(wgu_, dst, 2 * row, (const char*)wg.data + src, row, row, Fl), "upload gate");
                check(mf_write_2d(wgu_, dst + row, 2 * row, (const char*)wu.data + src, row, row, Fl), "upload up");
                check(mf_write_2d(wd_, e * d * Fl * esz, Fl * esz, (const char*)wd.data + (e * d * F + t * Fl) * esz,
                                  F * esz, Fl * esz, d),
                      "upload down");
            }
            own(wgu_);
            own(wd_);
        } else {
            // MoE: this rank's experts [lo, lo + n) (all of them without expert parallelism)
            const size_t e_lo = moe ? (size_t)c_.expert_lo() : 0, e_n = moe ? (size_t)c_.experts_local() : 1;
            const size_t nrows = moe ? e_n * F : Fl;
            const char* gsrc = (const char*)wg.data + (moe ? e_lo * F * row : t * Fl * row);
            const char* usrc = (const char*)wu.data + (moe ? e_lo * F * row : t * Fl * row);
            check(mf_alloc(2 * nrows * row, rank, &wgu_), "alloc gate/up");
            check(mf_write_2d(wgu_, 0, 2 * row, gsrc, row, row, nrows), "upload gate");
            check(mf_write_2d(wgu_, row, 2 * row, usrc, row, row, nrows), "upload up");
            own(wgu_);
            if (moe)
                own(wd_ = c_.ep() ? upload_rows(wd, e_lo * d, e_n * d, F * esz, rank) : upload_tensor(wd, rank));
            else
                own(wd_ = c_.tp_size == 1 ? upload_tensor(wd, rank)
                                          : upload_cols(wd, d, F * esz, t * Fl * esz, Fl * esz, rank));
        }
        const size_t k = moe ? (size_t)c_.n_active_experts : 1, ne = moe ? E : 1;
        read_bytes_ = moe ? fn.bytes + (wg.bytes / ne + wu.bytes / ne + wd.bytes / ne) * k
                          : fn.bytes + 2 * Fl * row + d * Fl * esz;
        // the k active experts are spread over the ranks (expert parallelism) or split in their rows
        if (moe && c_.tp_size > 1) read_bytes_ /= c_.tp_size;
        if (moe) {
            const TensorView& wr = f.tensor(p + "ffn_gate_inp.weight");
            expect_shape(wr, {E, d});
            expect_f32(wr);
            own(wr_ = upload_tensor(wr, rank));
            read_bytes_ += c_.tp_size > 1 ? wr.bytes / c_.tp_size : wr.bytes;  // replicated: each rank a share
        }
    }
    void cuda_forward(RunState& rs) override {
        const int d = c_.d_model, F = c_.d_ff;
        float* x = (float*)mf_ptr(rs.x);
        float* h = (float*)mf_ptr(rs.h);
        if (c_.n_experts == 0 && c_.tp_size > 1) {
            // receive the attention all-reduce (exchange 2l), send the FFN's (2l + 1)
            const int Fl = c_.ff_local();
            check(mf_allreduce_swiglu_matmul(h, (const float*)mf_ptr(rs.xb[0]), (float*)mf_ptr(rs.xb[1]),
                                             (const float*)mf_ptr(fn_), c_.rms_norm_eps, mf_ptr(wgu_), dtype_, Fl, d,
                                             rs.comm, 2 * layer_, rs.d_step, rs.stream),
                  "gate/up projection (all-reduce)");
            check(mf_matmul_push(h, mf_ptr(wd_), dtype_, d, Fl, rs.comm, 2 * layer_ + 1, rs.d_step, rs.stream),
                  "down projection (all-reduce send)");
            return;
        }
        if (c_.n_experts == 0) {
            check(mf_swiglu_matmul(h, x, (const float*)mf_ptr(fn_), c_.rms_norm_eps, mf_ptr(wgu_), dtype_, F, d,
                                   rs.stream),
                  "gate/up projection");
            check(mf_matmul_residual(x, h, mf_ptr(wd_), dtype_, d, F, rs.stream), "down projection");
            return;
        }
        const int k = c_.n_active_experts;
        int* ids = (int*)mf_ptr(rs.expert_ids) + (size_t)layer_ * k;
        float* w = (float*)mf_ptr(rs.expert_w) + (size_t)layer_ * k;
        if (c_.moe_tp) {
            // receive the attention all-reduce (exchange 2l) in the router GEMV;
            // every expert on this rank's FFN rows; its partial goes out as 2l + 1
            const int Fl = c_.ff_local();
            float* xo = (float*)mf_ptr(rs.xb[1]);
            check(mf_allreduce_router_topk(ids, w, (float*)mf_ptr(rs.scores), (const float*)mf_ptr(rs.xb[0]), xo,
                                           (const float*)mf_ptr(fn_), c_.rms_norm_eps, (const float*)mf_ptr(wr_), d,
                                           c_.n_experts, k, rs.comm, 2 * layer_, rs.d_step, rs.stream),
                  "router (all-reduce)");
            check(mf_moe_swiglu(h, xo, (const float*)mf_ptr(fn_), c_.rms_norm_eps, mf_ptr(wgu_), dtype_, ids, k, Fl, d,
                                rs.stream),
                  "expert gate/up (rows of this rank)");
            check(mf_moe_down_push(h, mf_ptr(wd_), dtype_, ids, w, k, d, Fl, 0, c_.n_experts, rs.comm,
                                   2 * layer_ + 1, rs.d_step, rs.stream),
                  "expert down (all-reduce send)");
            return;
        }
        if (c_.ep()) {
            // router on every rank (identical ids); this rank's experts only; their
            // weighted sum goes out as exchange `layer`, received by the next layer
            float* xl = (float*)mf_ptr(rs.xb[layer_ & 1]);
            check(mf_router_topk(ids, w, (float*)mf_ptr(rs.scores), xl, (const float*)mf_ptr(fn_), c_.rms_norm_eps,
                                 (const float*)mf_ptr(wr_), d, c_.n_experts, k, rs.stream),
                  "router");
            check(mf_moe_swiglu_ep(h, xl, (const float*)mf_ptr(fn_), c_.rms_norm_eps, mf_ptr(wgu_), dtype_, ids, k, F,
                                   d, c_.expert_lo(), c_.experts_local(), rs.stream),
                  "expert gate/up (local experts)");
            check(mf_moe_down_push(h, mf_ptr(wd_), dtype_, ids, w, k, d, F, c_.expert_lo(), c_.experts_local(),
                                   rs.comm, layer_, rs.d_step, rs.stream),
                  "expert down (all-reduce send)");
            return;
        }
        check(mf_moe_ffn(x, h, (const float*)mf_ptr(fn_), c_.rms_norm_eps, (const float*)mf_ptr(wr_), mf_ptr(wgu_),
                         mf_ptr(wd_), dtype_, (float*)mf_ptr(rs.scores), ids, w, d, F, c_.n_experts, k, rs.stream),
              "router + experts");
    }

    // dense FFN for n prompt tokens: pre-norm, gate/up GEMM with the SwiGLU
    // epilogue, down GEMM + residual
    void prefill_forward(RunState& rs, int n, int pos0) override {
        if (c_.n_experts > 0) {
            moe_prefill(rs, n);
            return;
        }
        const int d = c_.d_model, F = c_.ff_local();
        float* X = (float*)mf_ptr(rs.pf_x);
        void *hi = mf_ptr(rs.pf_hi), *lo = mf_ptr(rs.pf_lo), *hhi = mf_ptr(rs.pf_hhi), *hlo = mf_ptr(rs.pf_hlo);
        check(mf_prefill_norm_split(hi, lo, nullptr, X, (const float*)mf_ptr(fn_), c_.rms_norm_eps, d, n, rs.stream),
              "prefill ffn norm");
        if (!wgu_s_.hi) {
            check(mf_prefill_gemm(nullptr, 0, hi, lo, mf_ptr(wgu_), n, 2 * F, d, MF_PREFILL_SWIGLU, hhi, hlo,
                                  rs.stream),
                  "prefill gate/up projection");
        } else {
            // fp32 weights: both products summed in fp32 before the SwiGLU
            float* gu = (float*)mf_ptr(rs.pf_gu);
            prefill_gemm(gu, 2 * F, hi, lo, wgu_, wgu_s_, n, 2 * F, d, MF_PREFILL_STORE, rs.stream,
                         "prefill gate/up projection");
            check(mf_prefill_swiglu_split(hhi, hlo, gu, n, F, rs.stream), "prefill swiglu");
        }
        if (c_.tp_size == 1) {
            prefill_gemm(X, d, hhi, hlo, wd_, wd_s_, n, d, F, MF_PREFILL_RESID, rs.stream, "prefill down projection");
        } else {
            float* part = prefill_exchange_slot(rs);
            prefill_gemm(part, d, hhi, hlo, wd_, wd_s_, n, d, F, MF_PREFILL_STORE, rs.stream,
                         "prefill down projection (partial)");
            prefill_exchange(rs, X, n, d);
        }
    }
    // MoE FFN for n prompt tokens (module.cpp:440-476 per token): fp32 router
    // + top-k per token, tokens grouped by expert, grouped tcgen05 GEMMs
    // (gate/up with the SwiGLU epilogue, down), then every token adds its
    // experts' outputs in slot order
    void moe_prefill(RunState& rs, int n) {
        // (F: this rank's rows of every expert under tensor parallelism)
        const int d = c_.d_model, F = c_.ff_local(), E = c_.n_experts, k = c_.n_active_experts;
        const int El = c_.experts_local();  // under expert parallelism this rank's experts only
        float* X = (float*)mf_ptr(rs.pf_x);
        float* xn = (float*)mf_ptr(rs.pf_xn);
        int* ids = (int*)mf_ptr(rs.pf_ids) + (size_t)layer_ * rs.pf_cap * k;
        float* wts = (float*)mf_ptr(rs.pf_wts) + (size_t)layer_ * rs.pf_cap * k;
        int* grows = (int*)mf_ptr(rs.pf_grows);
        int* gtiles = (int*)mf_ptr(rs.pf_gtiles);
        int* pos = (int*)mf_ptr(rs.pf_pos);
        check(mf_prefill_norm_split(mf_ptr(rs.pf_hi), mf_ptr(rs.pf_lo), xn, X, (const float*)mf_ptr(fn_),
                                    c_.rms_norm_eps, d, n, rs.stream),
              "prefill ffn norm");
        check(mf_prefill_moe_route(ids, wts, xn, (const float*)mf_ptr(wr_), n, d, E, k, rs.stream), "prefill router");
        check(mf_prefill_moe_group(ids, n, k, c_.expert_lo(), El, grows, gtiles, pos, rs.stream),
              "prefill expert grouping");
        check(mf_prefill_moe_gather(mf_ptr(rs.pf_ghi), mf_ptr(rs.pf_glo), xn, pos, n, k, d, rs.stream),
              "prefill expert operands");
        check(mf_prefill_gemm_grouped(nullptr, 0, mf_ptr(rs.pf_ghi), mf_ptr(rs.pf_glo), mf_ptr(wgu_), El, n * k,
                                      2 * F, d, grows, gtiles, MF_PREFILL_SWIGLU, mf_ptr(rs.pf_mhi),
                                      mf_ptr(rs.pf_mlo), rs.stream),
              "prefill expert gate/up");
        check(mf_prefill_gemm_grouped((float*)mf_ptr(rs.pf_y), d, mf_ptr(rs.pf_mhi), mf_ptr(rs.pf_mlo), mf_ptr(wd_),
                                      El, n * k, d, F, grows, gtiles, MF_PREFILL_STORE, nullptr, nullptr, rs.stream),
              "prefill expert down");
        if (c_.tp_size == 1) {
            check(mf_prefill_moe_combine(X, X, (const float*)mf_ptr(rs.pf_y), pos, wts, n, k, d, rs.stream),
                  "prefill expert combine");
        } else {
            // this rank's slots from zero into the exchange slot; the ranks'
            // partials are summed into the residual (rank order)
            float* part = prefill_exchange_slot(rs);
            check(mf_prefill_moe_combine(part, nullptr, (const float*)mf_ptr(rs.pf_y), pos, wts, n, k, d, rs.stream),
                  "prefill expert combine (partial)");
            prefill_exchange(rs, X, n, d);
        }
        (void)E;
        // the last prompt token's routing, where the decode step keeps it
        check(mf_copy(rs.expert_ids, (size_t)layer_ * k * 4, rs.pf_ids,
                      ((size_t)layer_ * rs.pf_cap + (size_t)(n - 1)) * k * 4, (size_t)k * 4),
              "prefill expert ids");
        check(mf_copy(rs.expert_w, (size_t)layer_ * k * 4, rs.pf_wts,
                      ((size_t)layer_ * rs.pf_cap + (size_t)(n - 1)) * k * 4, (size_t)k * 4),
              "prefill expert weights");
    }
    void split_for_prefill(int rank) override {
        if (dtype_ != MF_F32 || c_.n_experts > 0 || wgu_s_.hi) return;
        const size_t d = c_.d_model, Fl = (size_t)c_.ff_local();
        wgu_s_ = split_weight(wgu_, 2 * Fl * d, rank);
        wd_s_ = split_weight(wd_, d * Fl, rank);
        for (mf_buf* b : {wgu_s_.hi, wgu_s_.lo, wd_s_.hi, wd_s_.lo}) own(b);
    }

private:
    const Config& c_;
    int layer_;
    int dtype_ = MF_BF16;
    mf_buf *fn_ = nullptr, *wgu_ = nullptr, *wd_ = nullptr, *wr_ = nullptr;
    SplitWeight wgu_s_, wd_s_;  // fp32 models: prefill copies
};

// Qwen3FinalRMSNorm (module.cpp:105-138) + Qwen3LMHead (module.cpp:46-103):
// the final norm is applied in the lm_head prologue.
class Qwen3LMHead : public BaseLayer {
public:
    Qwen3LMHead(const Config& c, const Qwen3Embed* embed) : c_(c), embed_(embed) {}
    void upload(const GGUFFile& f, int rank) override {
        const TensorView& on = f.tensor("output_norm.weight");
        expect_shape(on, {(uint64_t)c_.d_model});
        expect_f32(on);
        own(on_ = upload_tensor(on, rank));
        // under tensor parallelism this rank's vocabulary rows
        const size_t V0 = c_.vocab_offset(), Vl = c_.vocab_local();
        if (c_.untied_head) {
            const TensorView& t = f.tensor("output.weight");
            expect_shape(t, {c_.vocab_size, (uint64_t)c_.d_model});
            dtype_ = mf_dtype(t.dtype);
            const size_t rowb = t.bytes / c_.vocab_size;
            own(w_ = c_.tp_size == 1 ? upload_tensor(t, rank) : upload_rows(t, V0, Vl, rowb, rank));
            head_bytes_ = Vl * rowb;
        } else {
            const TensorView& t = f.tensor("token_embd.weight");
            w_ = embed_->weight();  // tied (src/models/qwen3/model.cpp:79-85); the table stays whole
            dtype_ = embed_->dtype();
            const size_t rowb = t.bytes / c_.vocab_size;
            w_off_ = V0 * rowb;
            head_bytes_ = Vl * rowb;
        }
        norm_bytes_ = on.bytes;
        read_bytes_ = head_bytes_ + norm_bytes_;
    }
    void cuda_forward(RunState& rs) override {
        if (!rs.compute_logits) return;
        if (c_.tp_size > 1) {
            // receive the last all-reduce (the last layer's down projection or
            // experts); greedy id agreed over ranks; full logits gathered when
            // the host wants them
            const int L = c_.n_layers;
            const int seq = c_.ep() ? L - 1 : 2 * L - 1;
            mf_buf* res = c_.ep() ? rs.xb[(L - 1) & 1] : rs.xb[1];
            mf_buf* out = c_.ep() ? rs.xb[L & 1] : rs.xb[0];
            check(mf_allreduce_lm_head((float*)mf_ptr(rs.logits), (const float*)mf_ptr(res), (float*)mf_ptr(out),
                                       (const float*)mf_ptr(on_), c_.rms_norm_eps, (const char*)mf_ptr(w_) + w_off_,
                                       dtype_, (int)c_.vocab_local(), c_.d_model, (int)c_.vocab_offset(), rs.d_step,
                                       mf_ptr(rs.lmh_ws), rs.host_logits ? 1 : 0, rs.comm, seq, rs.stream),
                  "lm_head (all-reduce)");
            return;
        }
        check(mf_lm_head((float*)mf_ptr(rs.logits), (const float*)mf_ptr(rs.x), (const float*)mf_ptr(on_),
                         c_.rms_norm_eps, mf_ptr(w_), dtype_, (int)c_.vocab_size, c_.d_model, 0, rs.d_step,
                         mf_ptr(rs.lmh_ws), rs.stream),
              "lm_head");
    }
    size_t head_bytes() const { return head_bytes_; }
    size_t norm_bytes() const { return norm_bytes_; }

private:
    const Config& c_;
    const Qwen3Embed* embed_;
    int dtype_ = MF_BF16;
    mf_buf *on_ = nullptr, *w_ = nullptr;
    size_t w_off_ = 0;  // byte offset of this rank's first row in w_ (tied head)
    size_t head_bytes_ = 0, norm_bytes_ = 0;
};

}  // namespace

BaseLayer::~BaseLayer() {
    for (mf_buf* b : bufs_) mf_release(b);
}

void BaseLayer::prefill_forward(RunState&, int, int) {}  // layers without prefill work (the lm_head)

Config Config::from_gguf(const GGUFFile& f, const RunParams& rp) {
    Config c;
    const std::string arch = f.get_string("general.architecture");
    if (arch != "qwen3") throw std::runtime_error("unsupported architecture " + arch);
    const std::string p = arch + ".";
    c.model_max_seq_len = f.get_uint(p + "context_length");
    c.d_model = (int)f.get_uint(p + "embedding_length");
    c.n_layers = (int)f.get_uint(p + "block_count");
    c.n_heads = (int)f.get_uint(p + "attention.head_count");
    c.n_kv_heads = (int)f.get_uint(p + "attention.head_count_kv");
    const int dk = (int)f.get_uint(p + "attention.key_length");
    const int dv = (int)f.get_uint(p + "attention.value_length");
    if (dk != dv) throw std::runtime_error("key_length != value_length");
    c.d_head = dk;
    c.d_ff = (int)(f.has(p + "expert_feed_forward_length") ? f.get_uint(p + "expert_feed_forward_length")
                                                           : f.get_uint(p + "feed_forward_length"));
    c.rms_norm_eps = (float)f.get_float(p + "attention.layer_norm_rms_epsilon");
    c.d_rotary = c.d_head;  // src/base/config.cpp:308
    c.freq_base = (float)f.get_float(p + "rope.freq_base");
    c.n_experts = f.has(p + "expert_count") ? (int)f.get_uint(p + "expert_count") : 0;
    c.n_active_experts = f.has(p + "expert_used_count") ? (int)f.get_uint(p + "expert_used_count") : 0;
    if (c.n_active_experts > c.n_experts) throw std::runtime_error("expert_used_count > expert_count");
    const MetaValue* toks = f.get("tokenizer.ggml.tokens");
    if (!toks || toks->kind != MetaValue::ARRAY_STR) throw std::runtime_error("missing tokenizer.ggml.tokens");
    c.vocab_size = toks->strs.size();
    c.eos_token_id = (uint32_t)f.get_uint("tokenizer.ggml.eos_token_id");
    c.padding_token_id = (uint32_t)f.get_uint("tokenizer.ggml.padding_token_id");
    if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads != 0)
        throw std::runtime_error("head counts are inconsistent");
    c.num_iters = rp.num_iters;
    c.user_max_seq_len = rp.max_seq_len;
    if (c.user_max_seq_len == 0 || c.user_max_seq_len > c.model_max_seq_len)
        throw std::runtime_error("max_seq_len must be in [1, context_length]");
    c.top_k = rp.top_k;
    c.temp = rp.temp;
    c.top_p = rp.top_p;
    c.min_p = rp.min_p;
    c.penalty_pres = rp.penalty_pres;
    c.seed = rp.seed;
    c.weight_dtype = f.tensor("blk.0.attn_q.weight").dtype;
    c.untied_head = f.has_tensor("output.weight");
    c.head_dtype = f.tensor(c.untied_head ? "output.weight" : "token_embd.weight").dtype;
    return c;
}

namespace {
// Frames are captured per manager rank; every model instance owns a disjoint
// block of frame ids so two models on one device never replay each other's graphs.
// 0-2 forward, 3-4 chained decode, 5-6 logits after a batched prefill, 7-8 forward / prefill
// logits read back as top-k candidates
constexpr int kFrameKinds = 12;  // kinds 10 / 11: sampled chains (first frame uploads the record)
int next_frame_base() {
    static int next = 0;
    const int b = next;
    next += kFrameKinds;
    return b;
}
}  // namespace

Qwen3Model::Qwen3Model(const std::string& path, const RunParams& rp, int rank, int tp_rank, int tp_size)
    : path_(path), rp_(rp), rank_(rank), frame_base_(next_frame_base()) {
    if (file_.open(path) != 0) throw std::runtime_error("failed to load model file " + path + ": " + file_.error());
    cfg_ = Config::from_gguf(file_, rp);
    if (tp_size < 1 || tp_size > MF_TP_MAX || tp_rank < 0 || tp_rank >= tp_size)
        throw std::invalid_argument("tp_rank/tp_size out of range");
    if (tp_size > 1 && cfg_.n_experts > 0) {
        // tensor parallelism inside every expert when the KV heads and the
        // expert FFN rows divide over the ranks (MF_MOE_EP=1: expert parallelism)
        const char* ep_env = std::getenv("MF_MOE_EP");
        cfg_.moe_tp = !(ep_env && ep_env[0] == '1') && cfg_.n_kv_heads % tp_size == 0 &&
                      cfg_.d_ff % tp_size == 0 && (cfg_.d_ff / tp_size) % 16 == 0 && 2 * cfg_.n_layers <= 255;
        if (!cfg_.moe_tp && cfg_.n_experts % tp_size != 0)
            throw std::invalid_argument("expert_count is not divisible by the expert-parallel size");
        if (cfg_.n_layers > 255) throw std::invalid_argument("expert parallelism supports up to 255 layers");
    } else if (tp_size > 1) {
        if (cfg_.n_kv_heads % tp_size != 0)
            throw std::invalid_argument("n_kv_heads is not divisible by the tensor-parallel size");
        if (cfg_.d_ff % tp_size != 0) throw std::invalid_argument("d_ff is not divisible by the tensor-parallel size");
        if (2 * cfg_.n_layers > 255) throw std::invalid_argument("tensor parallelism supports up to 127 layers");
    }
    cfg_.tp_rank = tp_rank;
    cfg_.tp_size = tp_size;
    reset_sampler();
    build_layers();
}

Qwen3Model::~Qwen3Model() {
    if (device_ == DeviceType::CUDA) {
        mf_sync(rank_);
        mf_drop_frames(rank_, frame_base_, frame_base_ + kFrameKinds - 1);
    }
    if (rs_.comm) mf_comm_destroy(rs_.comm);
    layers_.clear();
    for (mf_buf* b : state_bufs_) mf_release(b);
    if (rs_.h_logits) mf_host_free(rs_.h_logits);
    if (rs_.h_topk) mf_host_free(rs_.h_topk);
}

void Qwen3Model::reset_sampler() {
    SamplerParams sp;
    sp.vocab_size = cfg_.vocab_size;
    sp.top_k = cfg_.top_k;
    sp.temp = cfg_.temp;
    sp.top_p = cfg_.top_p;
    sp.min_p = cfg_.min_p;
    sp.penalty_pres = cfg_.penalty_pres;
    sp.seed = cfg_.seed;
    sampler_ = std::make_unique<Sampler>(sp);
}

void Qwen3Model::build_layers() {
    auto embed = std::make_unique<Qwen3Embed>(cfg_);
    Qwen3Embed* e = embed.get();
    layers_.push_back(std::move(embed));
    for (int i = 0; i < cfg_.n_layers; ++i) {
        layers_.push_back(std::make_unique<Qwen3GQA>(cfg_, i));
        layers_.push_back(std::make_unique<Qwen3MoE>(cfg_, i));
    }
    layers_.push_back(std::make_unique<Qwen3LMHead>(cfg_, e));
}

void Qwen3Model::set_device(DeviceType d) {
    if (d == device_) return;
    if (d != DeviceType::CUDA) throw std::runtime_error("this runtime moves models to CUDA only");
    for (auto& l : layers_) l->upload(file_, rank_);
    alloc_state();
    device_ = d;
}

void Qwen3Model::set_kv_dtype(int dtype) {
    if (dtype != MF_F32 && dtype != MF_BF16) throw std::invalid_argument("KV cache dtype must be f32 or bf16");
    if (device_ == DeviceType::CUDA) throw std::logic_error("set the KV cache dtype before moving the model to CUDA");
    kv_dtype_ = dtype;
}

void Qwen3Model::alloc_state() {
    const Config& c = cfg_;
    RunState& rs = rs_;
    rs.rank = rank_;
    rs.stream = mf_stream(rank_);
    auto alloc = [&](size_t bytes, const char* what) {
        mf_buf* b = nullptr;
        check(mf_alloc(bytes < 16 ? 16 : bytes, rank_, &b), what);
        state_bufs_.push_back(b);
        return b;
    };
    const size_t S = c.user_max_seq_len;
    const int k = std::max(c.n_active_experts, 1);
    const int Hl = c.heads_local(), Hkvl = c.kv_heads_local();
    rs.x = alloc((size_t)c.d_model * 4, "x");
    if (c.tp_size > 1) {
        rs.xb[0] = rs.x;
        rs.xb[1] = alloc((size_t)c.d_model * 4, "x (all-reduce ping-pong)");
    }
    rs.qkv = alloc((size_t)(Hl + 2 * Hkvl) * c.d_head * 4, "qkv");
    rs.att = alloc((size_t)Hl * c.d_head * 4, "att_out");
    rs.h = alloc((size_t)(c.n_experts > 0 ? c.d_ff : c.ff_local()) * k * 4, "hidden");
    rs.logits = alloc(c.vocab_size * 4, "logits");
    rs.scores = alloc((size_t)std::max(c.n_experts, 1) * 4, "moe_scores");
    rs.expert_ids = alloc((size_t)c.n_layers * k * 4, "active_experts");
    rs.expert_w = alloc((size_t)c.n_layers * k * 4, "active_experts_weights");
    rs.kv_dtype = kv_dtype_;
    rs.kv_elem = kv_dtype_ == MF_BF16 ? 2 : 4;
    rs.kv_layer_elems = (size_t)Hkvl * S * c.d_head;
    rs.k_cache = alloc(rs.kv_layer_elems * c.n_layers * rs.kv_elem, "k_cache");
    rs.v_cache = alloc(rs.kv_layer_elems * c.n_layers * rs.kv_elem, "v_cache");
    {
        std::vector<float> tab(S * (size_t)c.d_rotary);
        check(mf_rope_table(tab.data(), (int)S, c.d_rotary, c.freq_base), "rope table");
        rs.rope = alloc(tab.size() * 4, "rope table");
        check(mf_write(rs.rope, 0, tab.data(), tab.size() * 4), "upload rope table");
    }
    rs.attn_split = mf_attn_default_split(Hkvl, (int)S);
    rs.attn_ws = alloc(mf_attn_workspace_bytes(Hl, Hkvl, c.d_head, rs.attn_split), "attn workspace");
    rs.lmh_ws = alloc(mf_lm_head_workspace_bytes(), "lm_head workspace");
    check(mf_step_state(rank_, &rs.h_step, &rs.d_step), "step state");
    void* hl = nullptr;
    check(mf_host_alloc(c.vocab_size * 4, &hl), "pinned logits");
    rs.h_logits = (float*)hl;
    rs.topk_ids = alloc(kTopkMax * 4, "top-k ids");
    rs.topk_vals = alloc(kTopkMax * 4, "top-k logits");
    rs.topk_ws_bytes = mf_topk_workspace_bytes((int)c.vocab_size, kTopkMax);
    rs.topk_ws = alloc(rs.topk_ws_bytes, "top-k workspace");
    rs.smp_draws = alloc((S + 1) * 4, "sampling draws");
    rs.smp_ids = alloc((S + 1) * 4, "sampled ids");
    rs.smp_flags = alloc(16, "sampling flags");
    check(mf_host_alloc(2 * kTopkMax * 4, &rs.h_topk), "pinned top-k");
    rs.kv_bytes_per_pos = 2ull * c.n_layers * Hkvl * c.d_head * rs.kv_elem;
    if (c.tp_size > 1) {
        // dense models also get two bulk slots of [prompt chunk rows, d] for the batched prefill
        rs.pf_bulk_rows = (int)std::min<size_t>(c.user_max_seq_len, (size_t)kPrefillChunk);
        const size_t bulk = (size_t)rs.pf_bulk_rows * ((c.d_model + 3) / 4 * 4);
        check(mf_comm_create_ex(rank_, c.tp_rank, c.tp_size, (c.d_model + 3) / 4 * 4, (int)c.vocab_size, bulk,
                                &rs.comm),
              "tensor-parallel exchange");
        rs.zero_d = alloc((size_t)c.d_model * 4, "zero partial");
    }
}

void Qwen3Model::comm_handle(void* out, size_t n) const {
    if (!rs_.comm) throw std::runtime_error("no tensor-parallel exchange (tp_size 1, or set_device(CUDA) first)");
    check(mf_comm_handle(rs_.comm, out, n), "exchange handle");
}

void Qwen3Model::comm_connect(const void* handles, size_t n) {
    if (!rs_.comm) throw std::runtime_error("no tensor-parallel exchange (tp_size 1, or set_device(CUDA) first)");
    check(mf_comm_connect(rs_.comm, handles, n), "exchange connect");
}

int Qwen3Model::comm_status(int* status) {
    if (!rs_.comm) {
        *status = 0;
        return MF_OK;
    }
    return mf_comm_status(rs_.comm, status, 1);
}

bool Qwen3Model::prefill_supported() const {
    if (device_ != DeviceType::CUDA) return false;
    // MoE: bf16 experts, up to 256 experts (a multiple of 4), k <= 32; one GPU
    // or expert parallelism
    if (cfg_.n_experts != 0 && (cfg_.weight_dtype != DataType::BF16 || cfg_.n_experts % 4 != 0 ||
                                cfg_.n_experts > 256 || cfg_.n_active_experts > 32))
        return false;
    if (cfg_.tp_size > 1 && (rs_.pf_bulk_rows <= 0 || !rs_.comm || cfg_.d_model % 4 != 0)) return false;
    // bf16 weights directly; fp32 weights through bf16 hi/lo copies (two products per GEMM)
    if ((cfg_.weight_dtype != DataType::BF16 && cfg_.weight_dtype != DataType::F32) || cfg_.d_head != 128 ||
        cfg_.d_model % 8 != 0 || cfg_.d_ff % 8 != 0)
        return false;
    const int G = cfg_.n_heads / cfg_.n_kv_heads;
    return G == 1 || G == 2 || G == 4 || G == 8 || G == 16;
}

void Qwen3Model::alloc_prefill(int rows) {
    if (rs_.pf_cap >= rows) return;
    RunState& rs = rs_;
    for (mf_buf** b : {&rs.pf_x, &rs.pf_hi, &rs.pf_lo, &rs.pf_hhi, &rs.pf_hlo, &rs.pf_qkv, &rs.pf_q, &rs.pf_tok,
                       &rs.pf_att, &rs.pf_gu, &rs.pf_xn, &rs.pf_ids, &rs.pf_wts, &rs.pf_grows, &rs.pf_gtiles,
                       &rs.pf_pos, &rs.pf_ghi, &rs.pf_glo, &rs.pf_mhi, &rs.pf_mlo, &rs.pf_y}) {
        if (*b) {
            state_bufs_.erase(std::find(state_bufs_.begin(), state_bufs_.end(), *b));
            mf_release(*b);
            *b = nullptr;
        }
    }
    const Config& c = cfg_;
    auto alloc = [&](size_t bytes, const char* what) {
        mf_buf* b = nullptr;
        check(mf_alloc(bytes < 16 ? 16 : bytes, rank_, &b), what);
        state_bufs_.push_back(b);
        return b;
    };
    const size_t R = (size_t)rows, qd = (size_t)c.n_heads * c.d_head;
    const size_t wide = std::max<size_t>({(size_t)c.d_model, qd});
    rs.pf_x = alloc(R * c.d_model * 4, "prefill residual");
    rs.pf_hi = alloc(R * wide * 2, "prefill operand hi");
    rs.pf_lo = alloc(R * wide * 2, "prefill operand lo");
    rs.pf_hhi = alloc(R * c.d_ff * 2, "prefill ffn hi");
    rs.pf_hlo = alloc(R * c.d_ff * 2, "prefill ffn lo");
    rs.pf_qkv = alloc(R * (qd + 2ull * c.n_kv_heads * c.d_head) * 4, "prefill qkv");
    rs.pf_q = alloc(R * qd * 4, "prefill queries");
    rs.pf_tok = alloc(R * 4, "prefill token ids");
    if (c.n_experts > 0) {
        const size_t k = c.n_active_experts, E = c.n_experts;
        rs.pf_xn = alloc(R * c.d_model * 4, "prefill normalised rows");
        rs.pf_ids = alloc((size_t)c.n_layers * R * k * 4, "prefill expert ids");
        rs.pf_wts = alloc((size_t)c.n_layers * R * k * 4, "prefill expert weights");
        rs.pf_grows = alloc((E + 1) * 4, "prefill expert rows");
        rs.pf_gtiles = alloc((E + 1) * 4, "prefill expert tiles");
        rs.pf_pos = alloc(R * k * 4, "prefill grouped rows");
        rs.pf_ghi = alloc(R * k * c.d_model * 2, "prefill expert operands hi");
        rs.pf_glo = alloc(R * k * c.d_model * 2, "prefill expert operands lo");
        rs.pf_mhi = alloc(R * k * c.d_ff * 2, "prefill expert swiglu hi");
        rs.pf_mlo = alloc(R * k * c.d_ff * 2, "prefill expert swiglu lo");
        rs.pf_y = alloc(R * k * c.d_model * 4, "prefill expert outputs");
    }
    if (c.weight_dtype == DataType::F32) {
        rs.pf_gu = alloc(R * 2ull * c.ff_local() * 4, "prefill gate/up rows");
        for (auto& l : layers_) l->split_for_prefill(rank_);
    }
    const char* se = std::getenv("MF_PREFILL_SIMT_ATTN");
    rs.pf_simt_attn = se && se[0] == '1';
    if (!rs.pf_simt_attn) {
        // sized for the longest history: keys up to max_seq_len
        check(mf_prefill_attention_scratch(rows, (int)c.user_max_seq_len, c.n_heads, c.n_kv_heads,
                                           &rs.pf_att_bytes),
              "prefill attention scratch size");
        rs.pf_att = alloc(rs.pf_att_bytes, "prefill attention operands");
    }
    rs.pf_cap = rows;
}

bool Qwen3Model::prefill(const uint32_t* tokens, int n, int pos0, bool compute_logits, bool host_logits) {
    if (!prefill_supported()) return false;
    if (n <= 0) throw std::invalid_argument("empty prompt");
    if (pos0 < 0 || (size_t)pos0 + (size_t)n > cfg_.user_max_seq_len)
        throw std::runtime_error("prompt runs past max_seq_len");
    for (int i = 0; i < n; ++i)
        if (tokens[i] >= cfg_.vocab_size) throw std::runtime_error("token id outside the vocabulary");
    // MF_PREFILL_CHUNK overrides the rows per pass (smaller chunks exercise the history path)
    const char* ce = std::getenv("MF_PREFILL_CHUNK");
    const size_t want = (ce && std::atoi(ce) > 0) ? (size_t)std::atoi(ce) : (size_t)kPrefillChunk;
    int chunk = (int)std::min<size_t>(cfg_.user_max_seq_len, want);
    if (cfg_.tp_size > 1) chunk = std::min(chunk, rs_.pf_bulk_rows);  // rows one exchange slot holds
    alloc_prefill(std::min(chunk, n));
    int last_rows = 0;
    for (int c0 = 0; c0 < n; c0 += rs_.pf_cap) {
        const int nc = std::min(rs_.pf_cap, n - c0);
        check(mf_write(rs_.pf_tok, 0, tokens + c0, (size_t)nc * 4), "prefill token ids");
        for (size_t i = 0; i + 1 < layers_.size(); ++i) layers_[i]->prefill_forward(rs_, nc, pos0 + c0);
        last_rows = nc;
    }
    int st = 0;
    check(mf_prefill_status(&st, 1), "prefill status");
    if (st) throw WaitTimeout("a prefill kernel wait gave up (status " + std::to_string(st) + ")");
    if (rs_.comm) {
        check(mf_comm_status(rs_.comm, &st, 0), "exchange status");
        if (st) throw WaitTimeout("a prefill exchange wait gave up (status " + std::to_string(st) + ")");
    }
    // the last token's residual row feeds the decode lm_head (under tensor
    // parallelism the lm_head adds an all-reduce to it: see below)
    const int L = cfg_.n_layers;
    mf_buf* last = cfg_.tp_size == 1 ? rs_.x : (cfg_.ep() ? rs_.xb[(L - 1) & 1] : rs_.xb[1]);
    check(mf_copy(last, 0, rs_.pf_x, (size_t)(last_rows - 1) * cfg_.d_model * 4, (size_t)cfg_.d_model * 4),
          "prefill last row");
    rs_.cur_pos = pos0 + n - 1;
    rs_.token_id = tokens[n - 1];
    if (!compute_logits) return true;
    rs_.compute_logits = true;
    rs_.host_logits = host_logits;
    rs_.h_step[0] = (int32_t)tokens[n - 1];
    rs_.h_step[1] = pos0 + n - 1;
    rs_.h_step[3] = 0;
    rs_.h_step[MF_STEP_FRAME] = next_frame();
    const int frame = frame_base_ + (host_logits ? (rs_.topk_k > 0 ? 8 : 6) : 5);
    const int rc = mf_begin_frame(rank_, frame);
    if (rc < 0) check(rc, "begin_frame");
    if (rc == MF_FRAME_RECORD) {
        try {
            if (cfg_.tp_size > 1) {
                // the sharded lm_head receives the last layer's all-reduce
                // (exchange 2L - 1, or L - 1 under expert parallelism) on top of
                // its residual; the residual is already complete, so every rank
                // sends a zero partial
                const bool ep = cfg_.ep();
                check(mf_allreduce((float*)mf_ptr(ep ? rs_.xb[L & 1] : rs_.xb[0]), (const float*)mf_ptr(last),
                                   (const float*)mf_ptr(rs_.zero_d), cfg_.d_model, rs_.comm, ep ? L - 1 : 2 * L - 1,
                                   rs_.d_step, rs_.stream),
                      "prefill zero all-reduce");
            }
            layers_.back()->cuda_forward(rs_);
            check(mf_copy_to_host_async(rs_.h_step, rs_.d_step, kStepReadback, rs_.stream), "step readback");
            if (host_logits) read_back_logits();
        } catch (...) {
            mf_abort_frame(rank_);
            throw;
        }
    }
    check(mf_end_frame(rank_), "end_frame");
    check_exchange_status();
    return true;
}

size_t Qwen3Model::read_bytes(bool with_logits) const {
    size_t b = 0;
    for (size_t i = 0; i + 1 < layers_.size(); ++i) b += layers_[i]->read_bytes();
    const auto* head = static_cast<const Qwen3LMHead*>(layers_.back().get());
    b += head->norm_bytes();
    if (with_logits) b += head->head_bytes();
    return b;
}

void Qwen3Model::issue_frame(bool readback) {
    for (auto& l : layers_) l->cuda_forward(rs_);
    if (rs_.device_sample) {
        // top_k + 1 candidates of the (gathered) logits, then the draw: the
        // record carries the sampled id into the next frame
        const float* src = (const float*)mf_ptr(rs_.logits);
        if (rs_.comm) {
            float* g = nullptr;
            check(mf_comm_gather_ptr(rs_.comm, &g), "gather buffer");
            src = g;
        }
        int* ids = (int*)mf_ptr(rs_.topk_ids);
        float* vals = (float*)mf_ptr(rs_.topk_vals);
        check(mf_topk(src, (int)cfg_.vocab_size, rs_.smp_top_k + 1, ids, vals, mf_ptr(rs_.topk_ws),
                      rs_.topk_ws_bytes, rs_.stream),
              "top-k candidates");
        check(mf_sample_step(ids, vals, rs_.smp_top_k, rs_.smp_temp, rs_.smp_top_p, rs_.smp_min_p,
                             (const float*)mf_ptr(rs_.smp_draws), rs_.smp_n_draws, rs_.d_step,
                             (int*)mf_ptr(rs_.smp_ids), (int*)mf_ptr(rs_.smp_flags), rs_.stream),
              "device sampling");
        return;
    }
    // the step record (greedy id) comes back with every host-driven frame;
    // logits (or their top-k candidates) when asked
    if (readback) check(mf_copy_to_host_async(rs_.h_step, rs_.d_step, kStepReadback, rs_.stream), "step readback");
    if (rs_.compute_logits && rs_.host_logits) read_back_logits();
}

void Qwen3Model::read_back_logits() {
    const float* src = (const float*)mf_ptr(rs_.logits);
    if (rs_.comm) {
        float* g = nullptr;
        check(mf_comm_gather_ptr(rs_.comm, &g), "gather buffer");
        src = g;  // all ranks' rows, complete when the lm_head kernel ends
    }
    if (rs_.topk_k > 0) {
        int* ids = (int*)mf_ptr(rs_.topk_ids);
        float* vals = (float*)mf_ptr(rs_.topk_vals);
        check(mf_topk(src, (int)cfg_.vocab_size, rs_.topk_k, ids, vals, mf_ptr(rs_.topk_ws), rs_.topk_ws_bytes,
                      rs_.stream),
              "top-k candidates");
        char* h = (char*)rs_.h_topk;
        check(mf_copy_to_host_async(h, ids, (size_t)rs_.topk_k * 4, rs_.stream), "top-k ids readback");
        check(mf_copy_to_host_async(h + kTopkMax * 4, vals, (size_t)rs_.topk_k * 4, rs_.stream),
              "top-k logits readback");
        return;
    }
    check(mf_copy_to_host_async(rs_.h_logits, src, cfg_.vocab_size * 4, rs_.stream), "logits readback");
}

void Qwen3Model::check_exchange_status() const {
    const int ds = rs_.h_step[MF_STEP_DSTATUS];
    if (ds != 0)
        throw WaitTimeout("a decode kernel's copy wait gave up (status " + std::to_string(ds) +
                          "); this frame's results are invalid");
    if (!rs_.comm) return;
    const int st = rs_.h_step[MF_STEP_STATUS];
    if (st != 0)
        throw WaitTimeout("a tensor-parallel exchange wait gave up (status " + std::to_string(st) +
                          "): a peer rank did not arrive in time; this frame's results are invalid");
}

void Qwen3Model::read_full_logits() {
    const float* src = (const float*)mf_ptr(rs_.logits);
    if (rs_.comm) {
        float* g = nullptr;
        check(mf_comm_gather_ptr(rs_.comm, &g), "gather buffer");
        src = g;
    }
    check(mf_copy_to_host_async(rs_.h_logits, src, cfg_.vocab_size * 4, rs_.stream), "logits readback");
    check(mf_sync(rank_), "sync");
}

void Qwen3Model::forward(uint32_t token, int pos, bool compute_logits, bool host_logits) {
    if (device_ != DeviceType::CUDA) throw std::runtime_error("call set_device(CUDA) first");
    if (pos < 0 || (size_t)pos >= cfg_.user_max_seq_len) throw std::runtime_error("position outside the KV cache");
    if (token >= cfg_.vocab_size) throw std::runtime_error("token id outside the vocabulary");
    rs_.cur_pos = pos;
    rs_.token_id = token;
    rs_.compute_logits = compute_logits;
    rs_.host_logits = compute_logits && host_logits;
    rs_.h_step[0] = (int32_t)token;
    rs_.h_step[1] = pos;
    rs_.h_step[3] = 0;
    rs_.h_step[MF_STEP_FRAME] = next_frame();  // every frame gets a new sequence number
    const int frame = frame_base_ + (compute_logits ? (host_logits ? (rs_.topk_k > 0 ? 7 : 2) : 0) : 1);
    const int rc = mf_begin_frame(rank_, frame);
    if (rc < 0) check(rc, "begin_frame");
    if (rc == MF_FRAME_RECORD) {
        try {
            issue_frame(true);
        } catch (...) {
            mf_abort_frame(rank_);
            throw;
        }
    }
    check(mf_end_frame(rank_), "end_frame");
    // the decode kernels (and the tensor-parallel lm_head) report waits that gave up in the step record
    check_exchange_status();
}

std::vector<uint32_t> Qwen3Model::generate(const std::vector<uint32_t>& prompt, size_t n_gen, const GenOptions& opt,
                                           GenStats* stats, std::vector<float>* margins) {
    if (prompt.empty()) throw std::runtime_error("empty prompt");
    if (prompt.size() > cfg_.user_max_seq_len) throw std::runtime_error("prompt longer than max_seq_len");
    const bool greedy = sampler_->greedy();
    const bool need_host = !greedy || opt.trace;
    // sampling needs only the top-k (id, logit) list when nothing else reads the
    // logits and there is no presence penalty (which changes the list with every
    // token); MF_HOST_TOPK=1 keeps the whole-vocabulary readback
    const char* ht = std::getenv("MF_HOST_TOPK");
    const bool cand = !greedy && !opt.trace && !margins && !opt.on_step && sampler_->penalty_pres() == 0.0f &&
                      sampler_->top_k() < (size_t)kTopkMax && !(ht && ht[0] == '1');
    // one candidate beyond top_k shows whether the k-th logit is tied with the next
    rs_.topk_k = cand ? (int)sampler_->top_k() + 1 : 0;
    // after the first token, sampled decode can run as a device chain (no host
    // round trip per token; one GPU); MF_DEVICE_SAMPLE=0 keeps the host loop
    const char* dsm = std::getenv("MF_DEVICE_SAMPLE");
    const bool dev_smp = cand && !opt.forced && cfg_.tp_size == 1 && !(dsm && dsm[0] == '0');
    struct TopkReset {
        int& k;
        ~TopkReset() { k = 0; }
    } topk_reset{rs_.topk_k};
    GenStats st;
    size_t model_bytes = 0, kv_bytes = 0;
    const double t0 = now_s();
    // prefill: batched on the tensor cores when the model allows it, else
    // token by token as the reference does (src/base/model.cpp:120-129)
    const bool batched = opt.batched_prefill && prompt.size() > 1 &&
                         prefill(prompt.data(), (int)prompt.size(), 0, true, need_host);
    for (size_t i = 0; i < prompt.size(); ++i) {
        const bool last = i + 1 == prompt.size();
        if (!batched) forward(prompt[i], (int)i, last, last && need_host);
        model_bytes += read_bytes(last);
        kv_bytes += rs_.kv_bytes_per_pos * (i + 1);
    }
    st.prefill_time = (float)(now_s() - t0);
    for (uint32_t t : prompt) sampler_->add_token(t);
    std::vector<uint32_t> tokens = prompt, out;
    const size_t num_iters = std::min(n_gen, cfg_.user_max_seq_len - tokens.size());
    size_t generated = 0;
    const double t1 = now_s();
    while (generated < num_iters) {
        uint32_t next;
        if (need_host) {
            const float* lg = rs_.h_logits;
            if (cand) {
                const char* h = (const char*)rs_.h_topk;
                const float* vals = (const float*)(h + kTopkMax * 4);
                if (Sampler::candidates_decisive(vals, (size_t)rs_.topk_k)) {
                    next = sampler_->sample_candidates((const uint32_t*)h, vals, sampler_->top_k());
                } else {
                    // equal logits among the candidates: the whole vocabulary decides
                    read_full_logits();
                    next = sampler_->sample(lg);
                }
            } else {
                next = sampler_->sample(lg);
            }
            if (margins) {
                float v1 = -INFINITY, v2 = -INFINITY;
                for (size_t i = 0; i < cfg_.vocab_size; ++i) {
                    if (lg[i] > v1) {
                        v2 = v1;
                        v1 = lg[i];
                    } else if (lg[i] > v2) {
                        v2 = lg[i];
                    }
                }
                margins->push_back(v1 - v2);
            }
            if (opt.on_step) opt.on_step(generated, lg, next);
        } else {
            next = device_argmax();
            if (opt.on_step) opt.on_step(generated, nullptr, next);
        }
        out.push_back(next);
        const uint32_t fed = opt.forced ? opt.forced[generated] : next;
        sampler_->add_token(fed);
        tokens.push_back(fed);
        generated++;
        if (generated == 1) st.ttft = st.prefill_time + (float)(now_s() - t1);
        if (opt.stop_at_eos && fed == cfg_.eos_token_id) break;
        if (dev_smp && generated == 1 && generated < num_iters) {
            // the rest as one device chain: frame j forwards the last id and samples
            // the next with draw j; one frame more than tokens, as the host loop
            // also forwards the last token. Equal logits among a step's candidates
            // fall back to the host loop from here (nothing consumed yet).
            const size_t rest = num_iters - generated;
            bool tie = false;
            const std::vector<uint32_t> ids = decode_sampled_chained(fed, (int)tokens.size() - 1, (int)rest + 1,
                                                                     sampler_->peek_draws(rest + 1), &tie);
            if (!tie) {
                size_t used = 0;
                for (size_t j = 0; j < rest; ++j) {
                    const uint32_t t = ids[j];
                    model_bytes += read_bytes(true);
                    kv_bytes += rs_.kv_bytes_per_pos * tokens.size();
                    out.push_back(t);
                    sampler_->add_token(t);
                    tokens.push_back(t);
                    generated++;
                    used++;
                    if (opt.stop_at_eos && t == cfg_.eos_token_id) break;
                }
                sampler_->skip_draws(used);
                model_bytes += read_bytes(true);
                kv_bytes += rs_.kv_bytes_per_pos * tokens.size();
                break;
            }
        }
        forward(fed, (int)tokens.size() - 1, true, need_host);
        model_bytes += read_bytes(true);
        kv_bytes += rs_.kv_bytes_per_pos * tokens.size();
    }
    const double dt = now_s() - t1;
    st.num_tokens_gen = (int)generated;
    st.decode_seconds = dt;
    st.throughput = dt > 0 ? (float)(generated / dt) : 0.f;
    st.bytes_read = (double)(model_bytes + kv_bytes);
    st.bandwidth = (float)(st.bytes_read / 1e9 / (dt + st.prefill_time));
    if (stats) *stats = st;
    return out;
}

GenStats Qwen3Model::benchmark(bool batched_prefill) {
    constexpr size_t kPP = 512, kTG = 128;
    if (cfg_.user_max_seq_len < kPP) throw std::runtime_error("benchmark needs max_seq_len >= 512");
    std::mt19937 gen(cfg_.seed);
    std::uniform_int_distribution<> distrib(0, (int)cfg_.vocab_size - 1);
    GenStats st;
    size_t model_bytes = 0, kv_bytes = 0;
    std::vector<uint32_t> pp(kPP);
    for (size_t i = 0; i < kPP; ++i) pp[i] = (uint32_t)distrib(gen);  // drawn in the loop's order
    const double t0 = now_s();
    const bool batched = batched_prefill && prefill(pp.data(), (int)kPP, 0, true, false);
    for (size_t i = 0; i < kPP; ++i) {
        if (!batched) forward(pp[i], (int)i, i == kPP - 1, false);
        model_bytes += read_bytes(true);  // as the reference counts it (lm_head included every step)
        kv_bytes += rs_.kv_bytes_per_pos * (i + 1);
    }
    st.prefill_time = (float)(now_s() - t0);
    st.ttft = st.prefill_time;
    const double t1 = now_s();
    for (size_t i = 0; i < kTG; ++i) {
        forward((uint32_t)distrib(gen), (int)i, true, false);
        model_bytes += read_bytes(true);
        kv_bytes += rs_.kv_bytes_per_pos * (i + 1);
    }
    const double dt = now_s() - t1;
    st.num_tokens_gen = (int)kTG;
    st.decode_seconds = dt;
    st.throughput = (float)(kTG / dt);
    st.bytes_read = (double)(model_bytes + kv_bytes);
    st.bandwidth = (float)(st.bytes_read / 1e9 / (dt + st.prefill_time));
    return st;
}

std::vector<uint32_t> Qwen3Model::decode_sampled_chained(uint32_t token, int start_pos, int n,
                                                        const std::vector<float>& draws, bool* tie) {
    if (device_ != DeviceType::CUDA) throw std::runtime_error("call set_device(CUDA) first");
    std::vector<uint32_t> out;
    if (n <= 0) return out;
    if (token >= cfg_.vocab_size) throw std::runtime_error("token id outside the vocabulary");
    if (start_pos < 0 || (size_t)(start_pos + n) > cfg_.user_max_seq_len)
        throw std::runtime_error("chained decode runs past max_seq_len");
    if (draws.size() < (size_t)n || draws.size() > cfg_.user_max_seq_len + 1)
        throw std::invalid_argument("one draw per sampled token");
    if (sampler_->greedy() || sampler_->penalty_pres() != 0.0f || sampler_->top_k() + 1 > (size_t)kTopkMax)
        throw std::invalid_argument("device sampling needs temperature > 0, no presence penalty, top_k < 64");
    check(mf_write(rs_.smp_draws, 0, draws.data(), draws.size() * 4), "upload draws");
    const int zero[4] = {0, 0, 0, 0};
    check(mf_write(rs_.smp_flags, 0, zero, sizeof(zero)), "clear sampling flags");
    rs_.device_sample = true;
    rs_.smp_top_k = (int)sampler_->top_k();
    rs_.smp_temp = rp_.temp;
    rs_.smp_top_p = rp_.top_p;
    rs_.smp_min_p = rp_.min_p;
    // the frames are captured once and replayed: their kernel arguments must
    // not change between calls, so the bound is the buffer's capacity
    rs_.smp_n_draws = (int)cfg_.user_max_seq_len + 1;
    struct Reset {
        RunState& rs;
        ~Reset() { rs.device_sample = false; }
    } reset{rs_};
    rs_.compute_logits = true;
    rs_.host_logits = true;  // under tensor parallelism the lm_head gathers every rank's logits
    rs_.h_step[0] = (int32_t)token;
    rs_.h_step[1] = start_pos;
    rs_.h_step[3] = 0;  // the lm_head does not advance the record; the sampling kernel does
    rs_.h_step[MF_STEP_FRAME] = next_frame();
    rs_.h_step[MF_STEP_SAMPLE] = 0;
    for (int i = 0; i < n; ++i) {
        const int frame = frame_base_ + (i == 0 ? 10 : 11);
        const int rc = mf_begin_frame_ex(rank_, frame, i == 0 ? 0 : MF_FRAME_NO_UPLOAD);
        if (rc < 0) check(rc, "begin_frame");
        if (rc == MF_FRAME_RECORD) {
            try {
                issue_frame(false);
            } catch (...) {
                mf_abort_frame(rank_);
                throw;
            }
        }
        check(mf_end_frame_async(rank_), "end_frame");
    }
    std::vector<int32_t> ids((size_t)n);
    int flags[4] = {0, 0, 0, 0};
    check(mf_copy_to_host_async(ids.data(), mf_ptr(rs_.smp_ids), (size_t)n * 4, rs_.stream), "sampled ids");
    check(mf_copy_to_host_async(flags, mf_ptr(rs_.smp_flags), sizeof(flags), rs_.stream), "sampling flags");
    check(mf_copy_to_host_async(rs_.h_step, rs_.d_step, MF_STEP_RECORD_BYTES, rs_.stream), "step readback");
    check(mf_sync(rank_), "sync");
    frame_seq_ = rs_.h_step[MF_STEP_FRAME];  // the sampling kernels advanced it on the device
    rs_.h_step[MF_STEP_SAMPLE] = 0;
    check_exchange_status();
    if (flags[0] & 6) throw std::runtime_error("device sampling failed (flags " + std::to_string(flags[0]) + ")");
    if (tie) *tie = (flags[0] & 1) != 0;
    out.assign(ids.begin(), ids.end());
    return out;
}

uint32_t Qwen3Model::decode_chained(uint32_t token, int start_pos, int n) {
    if (device_ != DeviceType::CUDA) throw std::runtime_error("call set_device(CUDA) first");
    if (n <= 0) return token;
    if (token >= cfg_.vocab_size) throw std::runtime_error("token id outside the vocabulary");
    if (start_pos < 0 || (size_t)(start_pos + n) > cfg_.user_max_seq_len)
        throw std::runtime_error("chained decode runs past max_seq_len");
    rs_.compute_logits = true;
    rs_.host_logits = false;
    rs_.h_step[0] = (int32_t)token;
    rs_.h_step[1] = start_pos;
    rs_.h_step[3] = 1;
    rs_.h_step[MF_STEP_FRAME] = next_frame();  // later frames advance it on the device
    for (int i = 0; i < n; ++i) {
        // frame kind 3 uploads the host record once; kind 4 continues from the
        // record the previous frame's lm_head advanced on the device
        const int frame = frame_base_ + (i == 0 ? 3 : 4);
        const int rc = mf_begin_frame_ex(rank_, frame, i == 0 ? 0 : MF_FRAME_NO_UPLOAD);
        if (rc < 0) check(rc, "begin_frame");
        if (rc == MF_FRAME_RECORD) {
            try {
                issue_frame(false);
            } catch (...) {
                mf_abort_frame(rank_);
                throw;
            }
        }
        check(mf_end_frame_async(rank_), "end_frame");
    }
    // the whole record: the frame number continues from the device's
    check(mf_copy_to_host_async(rs_.h_step, rs_.d_step, MF_STEP_RECORD_BYTES, rs_.stream), "step readback");
    check(mf_sync(rank_), "sync");
    const uint32_t last = (uint32_t)rs_.h_step[2];
    rs_.h_step[3] = 0;
    frame_seq_ = rs_.h_step[MF_STEP_FRAME];  // the chained lm_heads advanced it on the device
    check_exchange_status();
    return last;
}

int Qwen3Model::read_experts(int layer, int* ids, float* w) const {
    if (cfg_.n_experts == 0 || layer < 0 || layer >= cfg_.n_layers) return MF_E_INVALID;
    const size_t k = cfg_.n_active_experts;
    int rc = mf_read(rs_.expert_ids, (size_t)layer * k * 4, ids, k * 4);
    if (rc == MF_OK && w) rc = mf_read(rs_.expert_w, (size_t)layer * k * 4, w, k * 4);
    return rc;
}

int Qwen3Model::read_prefill_experts(int layer, int* ids, float* w, int n) const {
    if (cfg_.n_experts == 0 || layer < 0 || layer >= cfg_.n_layers || !rs_.pf_ids || n < 0 || n > rs_.pf_cap)
        return MF_E_INVALID;
    const size_t k = cfg_.n_active_experts, off = (size_t)layer * rs_.pf_cap * k * 4;
    int rc = ids ? mf_read(rs_.pf_ids, off, ids, (size_t)n * k * 4) : MF_OK;
    if (rc == MF_OK && w) rc = mf_read(rs_.pf_wts, off, w, (size_t)n * k * 4);
    return rc;
}

int Qwen3Model::read_kv(int layer, float* k, float* v, int n_pos) const {
    // returns rows [0, n_pos) in the reference's [pos][kv_head][d_head] order
    // (this rank's KV heads under tensor parallelism)
    if (layer < 0 || layer >= cfg_.n_layers || n_pos < 0 || (size_t)n_pos > cfg_.user_max_seq_len) return MF_E_INVALID;
    // (a bf16 cache is widened to fp32, exactly)
    const size_t D = cfg_.d_head, S = cfg_.user_max_seq_len, es = rs_.kv_elem;
    std::vector<uint8_t> tmp(rs_.kv_layer_elems * es);
    for (int which = 0; which < 2; ++which) {
        float* dst = which == 0 ? k : v;
        if (!dst) continue;
        int rc = mf_read(which == 0 ? rs_.k_cache : rs_.v_cache, (size_t)layer * tmp.size(), tmp.data(), tmp.size());
        if (rc) return rc;
        for (int p = 0; p < n_pos; ++p)
            for (int hh = 0; hh < cfg_.kv_heads_local(); ++hh) {
                float* out = dst + ((size_t)p * cfg_.kv_heads_local() + hh) * D;
                const uint8_t* src = tmp.data() + ((size_t)hh * S + p) * D * es;
                if (es == 4) {
                    std::memcpy(out, src, D * 4);
                } else {
                    for (size_t i = 0; i < D; ++i) {
                        uint16_t b;
                        std::memcpy(&b, src + 2 * i, 2);
                        const uint32_t u = (uint32_t)b << 16;
                        std::memcpy(out + i, &u, 4);
                    }
                }
            }
    }
    return MF_OK;
}

int Qwen3Model::read_x(float* x) const { return mf_read(rs_.x, 0, x, (size_t)cfg_.d_model * 4); }

}  // namespace minfer
