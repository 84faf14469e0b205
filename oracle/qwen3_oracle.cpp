/*
 * ORACLE — test infrastructure only. A CPU restatement of the reference's
 * Qwen3 token loop (dsuarez01/minfer CPU path) used to check the CUDA path and
 * as the "port" CPU baseline. Nothing in the product links or calls it.
 *
 * Parity pinning: the op functions are checked against the reference's own
 * known-answer tests (tests/src/cpu_ops/*.cpp, restated as golden vectors in
 * tests/golden/) and, bit for bit, against the reference's CPU code compiled
 * from its own sources (oracle/_ref) on the same inputs.
 *
 * Each function names the reference lines it restates. Floating-point
 * expressions are written in the reference's order; fused multiply-adds appear
 * only where the reference has them (the NEON vfmaq lanes of the GEMVs).
 * Compile with -std=c++17 (no FP contraction), as the reference build here.
 */
#include <fcntl.h>
#include <omp.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <numeric>
#include <random>
#include <string>
#include <unordered_set>
#include <vector>

namespace {

// ------------------------------------------------------------------ widening
float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// fp32 -> nearest bf16 (ties to even) -> fp32; finite inputs
float round_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

float f16_to_f32(uint16_t h) {
    // exact IEEE binary16 -> binary32
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while (!(man & 0x400));
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 0x1F) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

enum Dt { F32 = 0, F16 = 1, BF16 = 2 };

inline float wget(const void* w, int dt, size_t i) {
    if (dt == F32) return ((const float*)w)[i];
    if (dt == BF16) return bf16_to_f32(((const uint16_t*)w)[i]);
    return f16_to_f32(((const uint16_t*)w)[i]);
}

}  // namespace

extern "C" {

// src/ops/kernels.cpp:27-29
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

// src/ops/kernels.cpp:31-49
void orc_softmax(float* out, const float* in, int n) {
    float mx = -FLT_MAX;
    for (int i = 0; i < n; ++i)
        if (in[i] > mx) mx = in[i];
    float s = 0.0f;
    for (int i = 0; i < n; ++i) {
        out[i] = expf(in[i] - mx);
        s += out[i];
    }
    const float inv = 1.0f / s;
    for (int i = 0; i < n; ++i) out[i] *= inv;
}

// src/ops/kernels.cpp:51-65 (interleaved pairs) and :67-81 (NeoX pairs).
// The reference calls unqualified pow/cos/sin on floats; with <math.h> in
// scope (libc++ on its own platform, and the libstdc++ build of the reference
// here) those are the float overloads, so the whole rotation is float math.
// The reference build evaluates the interleaved rotation with separate
// roundings (no contraction), the NeoX one with the first product fused:
// each restatement reproduces its counterpart.
__attribute__((optimize("fp-contract=off")))
void orc_il_rope(float* out, const float* in, int head, int d_head, int d_rot, float base, int pos) {
    const float* hi = in + head * d_head;
    float* ho = out + head * d_head;
    for (int i = 0; i < d_rot / 2; ++i) {
        const float freq = 1.0f / powf(base, 2.0f * i / d_rot);
        const float angle = pos * freq;
        const float x0 = hi[2 * i];
        const float x1 = hi[2 * i + 1];
        ho[2 * i] = cosf(angle) * x0 - sinf(angle) * x1;
        ho[2 * i + 1] = sinf(angle) * x0 + cosf(angle) * x1;
    }
}

void orc_neox_rope(float* out, const float* in, int head, int d_head, int d_rot, float base, int pos) {
    const float* hi = in + head * d_head;
    float* ho = out + head * d_head;
    for (int i = 0; i < d_rot / 2; ++i) {
        const float freq = 1.0f / powf(base, 2.0f * i / d_rot);
        const float angle = pos * freq;
        const float x0 = hi[i];
        const float x1 = hi[i + d_rot / 2];
        ho[i] = cosf(angle) * x0 - sinf(angle) * x1;
        ho[i + d_rot / 2] = sinf(angle) * x0 + cosf(angle) * x1;
    }
}

// src/ops/kernels.cpp:83-110
void orc_attn(float* scores, float* out, const float* q, const float* k, const float* v, int seq_len, int d_head,
              int kv_dim) {
    const float scale = 1.0f / sqrtf((float)d_head);
    for (int p = 0; p < seq_len; ++p) {
        float s = 0.0f;
        for (int d = 0; d < d_head; ++d) s += q[d] * k[p * kv_dim + d];
        scores[p] = s * scale;
    }
    orc_softmax(scores, scores, seq_len);
    for (int d = 0; d < d_head; ++d) out[d] = 0.0f;
    for (int p = 0; p < seq_len; ++p) {
        const float sc = scores[p];
        for (int d = 0; d < d_head; ++d) out[d] += sc * v[p * kv_dim + d];
    }
}

// src/ops/kernels.cpp:351-365
void orc_rmsnorm(float* out, const float* in, const float* w, int dim, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < dim; ++i) ss += in[i] * in[i];
    const float rms = sqrtf(ss / dim + eps);
    const float inv = 1.0f / rms;
    for (int i = 0; i < dim; ++i) out[i] = inv * in[i] * w[i];
}

// src/ops/kernels.cpp:211-343: per row, 16 NEON lanes each accumulate
// fma(x[j+l], w[j+l], acc_l) over j += 16; the four float32x4 accumulators are
// added as (a0+a1)+(a2+a3) lane-wise and the result reduced pairwise
// ((t0+t1)+(t2+t3)). OpenMP over 16-row tiles like the reference.
void orc_matmul(float* out, const float* x, const void* w, int dt, size_t offset, int d_out, int d_in) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < (d_out + 15) / 16; ++t) {
        const int i_end = std::min(t * 16 + 16, d_out);
        for (int i = t * 16; i < i_end; ++i) {
            float acc[16] = {0};
            const size_t base = offset + (size_t)i * d_in;
            for (int j = 0; j < d_in; j += 16)
                for (int l = 0; l < 16; ++l) acc[l] = fmaf(x[j + l], wget(w, dt, base + j + l), acc[l]);
            float tt[4];
            for (int m = 0; m < 4; ++m) tt[m] = (acc[m] + acc[4 + m]) + (acc[8 + m] + acc[12 + m]);
            out[i] = (tt[0] + tt[1]) + (tt[2] + tt[3]);
        }
    }
}

// src/ops/kernels.cpp:113-139
void orc_route(const float* x, int* ids, float* weights, float* scores, const float* w_router, int d_model,
               int n_experts, int k) {
    orc_matmul(scores, x, w_router, F32, 0, n_experts, d_model);
    std::vector<bool> visited(n_experts, false);
    for (int i = 0; i < k; ++i) {
        int best = 0;
        float bs = -FLT_MAX;
        for (int j = 0; j < n_experts; ++j) {
            if (!visited[j] && scores[j] > bs) {
                best = j;
                bs = scores[j];
            }
        }
        ids[i] = best;
        weights[i] = bs;
        visited[best] = true;
    }
    orc_softmax(weights, weights, k);
}

// src/ops/kernels.cpp:153-187, src/base/types.cpp:14-38
void orc_embed(float* out, const void* w, int dt, uint32_t token, size_t d) {
    for (size_t i = 0; i < d; ++i) out[i] = wget(w, dt, (size_t)token * d + i);
}

}  // extern "C"

// =================================================================== model
namespace {

struct Tensor {
    const uint8_t* data = nullptr;
    int dt = F32;
    std::vector<uint64_t> shape;  // outermost first
    size_t bytes = 0;
};

// GGUF v3 reader (format of include/minfer/parsing/gguf.hpp; reading rules of
// src/parsing/gguf.cpp:145-242 restricted to what the model needs).
struct Gguf {
    void* map = nullptr;
    size_t size = 0;
    std::map<std::string, double> num;
    std::map<std::string, std::string> str;
    std::map<std::string, size_t> arr_len;
    std::map<std::string, Tensor> t;
    std::string err;

    ~Gguf() {
        if (map) munmap(map, size);
    }

    bool open(const char* path) {
        int fd = ::open(path, O_RDONLY);
        if (fd < 0) return fail("cannot open file");
        struct stat st;
        fstat(fd, &st);
        size = (size_t)st.st_size;
        map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (map == MAP_FAILED) {
            map = nullptr;
            return fail("mmap failed");
        }
        const uint8_t* p = (const uint8_t*)map;
        const uint8_t* end = p + size;
        auto rd = [&](void* dst, size_t n) {
            if ((size_t)(end - p) < n) throw 1;
            std::memcpy(dst, p, n);
            p += n;
        };
        auto u32 = [&]() { uint32_t v; rd(&v, 4); return v; };
        auto u64 = [&]() { uint64_t v; rd(&v, 8); return v; };
        auto s = [&]() {
            uint64_t n = u64();
            if (n > size) throw 1;
            std::string r(n, '\0');
            rd(&r[0], n);
            return r;
        };
        std::function<double(uint32_t)> scalar = [&](uint32_t ty) -> double {
            switch (ty) {
                case 0: { uint8_t v; rd(&v, 1); return v; }
                case 1: { int8_t v; rd(&v, 1); return v; }
                case 2: { uint16_t v; rd(&v, 2); return v; }
                case 3: { int16_t v; rd(&v, 2); return v; }
                case 4: return u32();
                case 5: { int32_t v; rd(&v, 4); return v; }
                case 6: { float v; rd(&v, 4); return v; }
                case 7: { uint8_t v; rd(&v, 1); return v; }
                case 10: return (double)u64();
                case 11: { int64_t v; rd(&v, 8); return (double)v; }
                case 12: { double v; rd(&v, 8); return v; }
                default: throw 1;
            }
        };
        try {
            if (u32() != 0x46554747u) return fail("bad magic");
            if (u32() != 3) return fail("not GGUF v3");
            const uint64_t nt = u64(), nkv = u64();
            for (uint64_t i = 0; i < nkv; ++i) {
                std::string key = s();
                const uint32_t ty = u32();
                if (ty == 8) {
                    str[key] = s();
                } else if (ty == 9) {
                    const uint32_t et = u32();
                    const uint64_t n = u64();
                    arr_len[key] = n;
                    for (uint64_t j = 0; j < n; ++j) {
                        if (et == 8) s();
                        else scalar(et);
                    }
                } else {
                    num[key] = scalar(ty);
                }
            }
            struct Info { std::string name; std::vector<uint64_t> ne; uint32_t ty; uint64_t off; };
            std::vector<Info> infos;
            for (uint64_t i = 0; i < nt; ++i) {
                Info in;
                in.name = s();
                const uint32_t nd = u32();
                for (uint32_t d = 0; d < nd; ++d) in.ne.push_back(u64());
                in.ty = u32();
                in.off = u64();
                infos.push_back(in);
            }
            uint64_t align = num.count("general.alignment") ? (uint64_t)num["general.alignment"] : 32;
            uint64_t pos = p - (const uint8_t*)map;
            uint64_t data0 = pos + (align - pos % align) % align;
            for (auto& in : infos) {
                Tensor tv;
                tv.dt = in.ty == 0 ? F32 : in.ty == 1 ? F16 : in.ty == 30 ? BF16 : -1;
                if (tv.dt < 0) return fail("unsupported tensor type");
                size_t n = 1;
                for (auto d : in.ne) n *= d;
                tv.bytes = n * (tv.dt == F32 ? 4 : 2);
                if (data0 + in.off + tv.bytes > size) return fail("tensor past end of file");
                tv.data = (const uint8_t*)map + data0 + in.off;
                tv.shape.assign(in.ne.rbegin(), in.ne.rend());
                t[in.name] = tv;
            }
        } catch (...) {
            return fail("truncated or malformed file");
        }
        return true;
    }
    bool fail(const char* m) {
        err = m;
        return false;
    }
};

}  // namespace

struct orc_model {
    Gguf f;
    // Config (src/base/config.cpp:277-337)
    int d, L, H, Hkv, D, F, E, K, V;
    float eps, base;
    uint32_t eos;
    size_t S;
    bool untied;
    // RunState (src/base/config.cpp:339-381)
    std::vector<float> x, xb, xb2, hb, hb2, q, k, v, att, att_out, kc, vc, scores, ew, logits;
    std::vector<int> experts;
    // per forward, per MoE layer: k expert ids (when recording)
    std::vector<int> rec_ids;
    std::vector<float> rec_w;
    bool record = false;
    // Emulation of the CUDA runtime's opt-in bf16 KV cache (the reference has
    // none): appended K/V rows rounded to bf16, nearest even, before use.
    bool kv_bf16 = false;
    // sampler state (src/base/sampler.cpp)
    size_t top_k;
    float temp, top_p, min_p, pres;
    std::unordered_set<uint32_t> seen;
    std::mt19937_64 rng;
    std::uniform_real_distribution<float> dist{0.0f, 1.0f};
    std::vector<float> sl, sp;
    std::vector<uint32_t> sidx;

    const Tensor& T(const std::string& n) { return f.t.at(n); }
};

extern "C" {

orc_model* orc_model_open(const char* path, size_t max_seq, size_t top_k, float temp, float top_p, float min_p,
                          float pres, int seed) {
    auto m = std::make_unique<orc_model>();
    if (!m->f.open(path)) {
        std::fprintf(stderr, "oracle: %s\n", m->f.err.c_str());
        return nullptr;
    }
    auto& n = m->f.num;
    const std::string a = "qwen3.";
    try {
        m->d = (int)n.at(a + "embedding_length");
        m->L = (int)n.at(a + "block_count");
        m->H = (int)n.at(a + "attention.head_count");
        m->Hkv = (int)n.at(a + "attention.head_count_kv");
        m->D = (int)n.at(a + "attention.key_length");
        m->F = (int)(n.count(a + "expert_feed_forward_length") ? n.at(a + "expert_feed_forward_length")
                                                                : n.at(a + "feed_forward_length"));
        m->E = n.count(a + "expert_count") ? (int)n.at(a + "expert_count") : 0;
        m->K = n.count(a + "expert_used_count") ? (int)n.at(a + "expert_used_count") : 0;
        m->eps = (float)n.at(a + "attention.layer_norm_rms_epsilon");
        m->base = (float)n.at(a + "rope.freq_base");
        m->eos = (uint32_t)n.at("tokenizer.ggml.eos_token_id");
        m->V = (int)m->f.arr_len.at("tokenizer.ggml.tokens");
    } catch (...) {
        std::fprintf(stderr, "oracle: missing metadata\n");
        return nullptr;
    }
    m->S = max_seq;
    m->untied = m->f.t.count("output.weight") != 0;
    const int d = m->d, qd = m->H * m->D, kvd = m->Hkv * m->D;
    m->x.resize(d); m->xb.resize(d); m->xb2.resize(d);
    m->hb.resize(m->F); m->hb2.resize(m->F);
    m->q.resize(qd); m->k.resize(kvd); m->v.resize(kvd);
    m->att.resize((size_t)m->H * max_seq); m->att_out.resize(qd);
    m->kc.assign((size_t)m->L * max_seq * kvd, 0.f);
    m->vc.assign((size_t)m->L * max_seq * kvd, 0.f);
    m->scores.resize(std::max(m->E, 1));
    m->experts.assign(std::max(m->K, 1), 0);
    m->ew.assign(std::max(m->K, 1), 1.0f);
    m->logits.resize(m->V);
    m->top_k = top_k; m->temp = temp; m->top_p = top_p; m->min_p = min_p; m->pres = pres;
    m->rng.seed((uint64_t)seed);
    m->sl.resize(m->V); m->sp.resize(m->V); m->sidx.resize(m->V);
    return m.release();
}

void orc_model_close(orc_model* m) { delete m; }

int orc_model_vocab(const orc_model* m) { return m->V; }

void orc_model_set_kv_bf16(orc_model* m, int on) { m->kv_bf16 = on != 0; }

void orc_model_record_experts(orc_model* m, int on) {
    m->record = on != 0;
    m->rec_ids.clear();
    m->rec_w.clear();
}

size_t orc_model_recorded(const orc_model* m, int* ids, float* w) {
    if (ids) std::memcpy(ids, m->rec_ids.data(), m->rec_ids.size() * sizeof(int));
    if (w) std::memcpy(w, m->rec_w.data(), m->rec_w.size() * sizeof(float));
    return m->rec_ids.size();
}

// One token through every layer (src/base/model.cpp:36-43 on the CPU path).
void orc_model_forward(orc_model* m, uint32_t token, int pos, int compute_logits) {
    const int d = m->d, H = m->H, Hkv = m->Hkv, D = m->D, F = m->F;
    const int kvd = Hkv * D;
    // Qwen3Embed::cpu_forward (src/models/qwen3/module.cpp:29-31)
    const Tensor& te = m->T("token_embd.weight");
    orc_embed(m->x.data(), te.data, te.dt, token, d);
    for (int l = 0; l < m->L; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        // Qwen3GQA::cpu_forward (src/models/qwen3/module.cpp:180-241)
        orc_rmsnorm(m->xb.data(), m->x.data(), (const float*)m->T(p + "attn_norm.weight").data, d, m->eps);
        const Tensor& wq = m->T(p + "attn_q.weight");
        const Tensor& wk = m->T(p + "attn_k.weight");
        const Tensor& wv = m->T(p + "attn_v.weight");
        orc_matmul(m->q.data(), m->xb.data(), wq.data, wq.dt, 0, H * D, d);
        orc_matmul(m->k.data(), m->xb.data(), wk.data, wk.dt, 0, kvd, d);
        orc_matmul(m->v.data(), m->xb.data(), wv.data, wv.dt, 0, kvd, d);
        const float* qn = (const float*)m->T(p + "attn_q_norm.weight").data;
        const float* kn = (const float*)m->T(p + "attn_k_norm.weight").data;
        for (int h = 0; h < H; ++h) orc_rmsnorm(m->q.data() + h * D, m->q.data() + h * D, qn, D, m->eps);
        for (int h = 0; h < H; ++h) orc_neox_rope(m->q.data(), m->q.data(), h, D, D, m->base, pos);
        for (int h = 0; h < Hkv; ++h) orc_rmsnorm(m->k.data() + h * D, m->k.data() + h * D, kn, D, m->eps);
        for (int h = 0; h < Hkv; ++h) orc_neox_rope(m->k.data(), m->k.data(), h, D, D, m->base, pos);
        const size_t co = (size_t)l * m->S * kvd + (size_t)pos * kvd;
        for (int i = 0; i < kvd; ++i) {
            m->kc[co + i] = m->kv_bf16 ? round_bf16(m->k[i]) : m->k[i];
            m->vc[co + i] = m->kv_bf16 ? round_bf16(m->v[i]) : m->v[i];
        }
        const int kv_mul = H / Hkv;
#pragma omp parallel for
        for (int h = 0; h < H; ++h) {
            const size_t ko = (size_t)l * m->S * kvd + (size_t)(h / kv_mul) * D;
            orc_attn(m->att.data() + (size_t)h * m->S, m->att_out.data() + h * D, m->q.data() + h * D,
                     m->kc.data() + ko, m->vc.data() + ko, pos + 1, D, kvd);
        }
        const Tensor& wo = m->T(p + "attn_output.weight");
        orc_matmul(m->xb.data(), m->att_out.data(), wo.data, wo.dt, 0, d, H * D);
        for (int i = 0; i < d; ++i) m->x[i] += m->xb[i];
        // Qwen3MoE::cpu_forward (src/models/qwen3/module.cpp:440-476)
        orc_rmsnorm(m->xb.data(), m->x.data(), (const float*)m->T(p + "ffn_norm.weight").data, d, m->eps);
        const bool moe = m->E > 0;
        if (moe) {
            orc_route(m->xb.data(), m->experts.data(), m->ew.data(), m->scores.data(),
                      (const float*)m->T(p + "ffn_gate_inp.weight").data, d, m->E, m->K);
            if (m->record) {
                m->rec_ids.insert(m->rec_ids.end(), m->experts.begin(), m->experts.begin() + m->K);
                m->rec_w.insert(m->rec_w.end(), m->ew.begin(), m->ew.begin() + m->K);
            }
        } else {
            m->experts[0] = 0;
            m->ew[0] = 1.0f;
        }
        const Tensor& wg = m->T(p + (moe ? "ffn_gate_exps.weight" : "ffn_gate.weight"));
        const Tensor& wu = m->T(p + (moe ? "ffn_up_exps.weight" : "ffn_up.weight"));
        const Tensor& wd = m->T(p + (moe ? "ffn_down_exps.weight" : "ffn_down.weight"));
        const int n = moe ? m->K : 1;
        for (int i = 0; i < n; ++i) {
            const size_t e = (size_t)m->experts[i];
            orc_matmul(m->hb.data(), m->xb.data(), wg.data, wg.dt, e * F * d, F, d);
            orc_matmul(m->hb2.data(), m->xb.data(), wu.data, wu.dt, e * F * d, F, d);
            for (int j = 0; j < F; ++j) m->hb[j] = orc_silu(m->hb[j]) * m->hb2[j];
            orc_matmul(m->xb2.data(), m->hb.data(), wd.data, wd.dt, e * d * F, d, F);
            for (int j = 0; j < d; ++j) m->x[j] += m->xb2[j] * m->ew[i];
        }
    }
    // Qwen3FinalRMSNorm + Qwen3LMHead (src/models/qwen3/module.cpp:54-79,113-126);
    // an untied `output.weight` is used when the file has one.
    orc_rmsnorm(m->x.data(), m->x.data(), (const float*)m->T("output_norm.weight").data, d, m->eps);
    if (compute_logits) {
        const Tensor& wl = m->T(m->untied ? "output.weight" : "token_embd.weight");
        orc_matmul(m->logits.data(), m->x.data(), wl.data, wl.dt, 0, m->V, d);
    }
}

const float* orc_model_logits(const orc_model* m) { return m->logits.data(); }

void orc_model_kv(const orc_model* m, int layer, int n_pos, float* k, float* v) {
    const size_t kvd = (size_t)m->Hkv * m->D;
    const size_t o = (size_t)layer * m->S * kvd;
    if (k) std::memcpy(k, m->kc.data() + o, n_pos * kvd * sizeof(float));
    if (v) std::memcpy(v, m->vc.data() + o, n_pos * kvd * sizeof(float));
}

void orc_sampler_add(orc_model* m, uint32_t tok) { m->seen.insert(tok); }

// Sampler::sample (src/base/sampler.cpp:34-117)
uint32_t orc_sample(orc_model* m, const float* logits) {
    const size_t V = (size_t)m->V;
    if (m->temp == 0.0f) return (uint32_t)(std::max_element(logits, logits + V) - logits);
    for (size_t i = 0; i < V; ++i) m->sl[i] = logits[i] - float(m->seen.count((uint32_t)i)) * m->pres;
    std::iota(m->sidx.begin(), m->sidx.end(), 0u);
    auto cmp = [&](size_t a, size_t b) { return m->sl[a] > m->sl[b]; };
    std::nth_element(m->sidx.begin(), m->sidx.begin() + m->top_k, m->sidx.end(), cmp);
    std::sort(m->sidx.begin(), m->sidx.begin() + m->top_k, cmp);
    size_t cut = m->top_k;
    float acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        m->sp[m->sidx[i]] = expf(m->sl[m->sidx[i]] - m->sl[m->sidx[0]]);
        acc += m->sp[m->sidx[i]];
    }
    for (size_t i = 0; i < cut; ++i) m->sp[m->sidx[i]] /= acc;
    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        acc += m->sp[m->sidx[i]];
        if (acc >= m->top_p) {
            cut = i + 1;
            break;
        }
    }
    if (m->min_p > 0.0f) {
        const float thr = m->sl[m->sidx[0]] + logf(m->min_p);
        for (size_t i = 0; i < cut; ++i) {
            if (m->sl[m->sidx[i]] < thr) {
                cut = i;
                break;
            }
        }
    }
    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        m->sp[m->sidx[i]] = expf((m->sl[m->sidx[i]] - m->sl[m->sidx[0]]) / m->temp);
        acc += m->sp[m->sidx[i]];
    }
    for (size_t i = 0; i < cut; ++i) m->sp[m->sidx[i]] /= acc;
    const float r = m->dist(m->rng);
    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        acc += m->sp[m->sidx[i]];
        if (acc >= r) return m->sidx[i];
    }
    return m->sidx[cut - 1];
}

// The first n numbers Sampler::sample draws: std::uniform_real_distribution<float>
// (0, 1) over std::mt19937_64(seed), one per sampled token
// (src/base/sampler.cpp:21-22, include/minfer/base/sampler.hpp:23-24).
void orc_uniform_draws(int seed, size_t n, float* out) {
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    for (size_t i = 0; i < n; ++i) out[i] = dist(rng);
}

// BaseModel::generate loop without the tokenizer (src/base/model.cpp:119-173),
// EOS ignored. out_ids[n_gen]; margins[n_gen] (top-1 minus top-2 logit of the
// logits each id was sampled from; may be NULL).
size_t orc_generate(orc_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t* out_ids,
                    float* margins) {
    for (size_t i = 0; i < n_prompt; ++i) orc_model_forward(m, prompt[i], (int)i, i + 1 == n_prompt);
    for (size_t i = 0; i < n_prompt; ++i) orc_sampler_add(m, prompt[i]);
    size_t ntok = n_prompt;
    const size_t iters = std::min(n_gen, m->S - n_prompt);
    for (size_t g = 0; g < iters; ++g) {
        const float* lg = m->logits.data();
        if (margins) {
            float v1 = -INFINITY, v2 = -INFINITY;
            for (int i = 0; i < m->V; ++i) {
                if (lg[i] > v1) {
                    v2 = v1;
                    v1 = lg[i];
                } else if (lg[i] > v2) {
                    v2 = lg[i];
                }
            }
            margins[g] = v1 - v2;
        }
        const uint32_t next = orc_sample(m, lg);
        orc_sampler_add(m, next);
        out_ids[g] = next;
        ntok++;
        orc_model_forward(m, next, (int)ntok - 1, 1);
    }
    return iters;
}

}  // extern "C"
