/*
 * minfer_model.h — C ABI of libminfer_host.so, the C++17 host runtime of the
 * Qwen3 token loop on CUDA (GGUF loader, Config/RunState, Qwen3 layers,
 * sampler, token loop) built over libmfcuda (minfer_cuda.h).
 *
 * It exposes what the reference's apps and tests reach through BaseModel
 * (include/minfer/base/model.hpp:17-41): construction from a GGUF file
 * (Qwen3Model::Qwen3Model, src/models/qwen3/model.cpp:9-86), set_device,
 * forward, generate and benchmark on token ids, and the tokenizer with its
 * chat template (Qwen3Tokenizer) for text, on the host (mf_tokenizer_*).
 *
 * Status codes are the MF_* codes of minfer_cuda.h; mf_last_error() returns
 * the message of the last failure (host-runtime failures included).
 */
#ifndef MINFER_MODEL_H
#define MINFER_MODEL_H

#include <stddef.h>
#include <stdint.h>

#include "minfer_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mf_model mf_model;

/* Message of the last failure of this library or of libmfcuda on this thread. */
int mf_host_last_error(char* buf, size_t n);

/* RunParams (include/minfer/base/config.hpp:37-51) */
typedef struct mf_run_params {
    size_t num_iters;
    size_t max_seq_len;
    size_t top_k;
    float temp;
    float top_p;
    float min_p;
    float penalty_pres;
    int seed;
} mf_run_params;

/* Config fields a caller needs (include/minfer/base/config.hpp:53-75) */
typedef struct mf_model_info {
    size_t vocab_size;
    size_t max_seq_len;
    int d_model, n_layers, n_heads, n_kv_heads, d_head, d_ff, n_experts, n_active_experts;
    int weight_dtype; /* MF_F32 / MF_F16 / MF_BF16 */
    int untied_head;
    uint32_t eos_token_id;
    float rms_norm_eps, freq_base;
    size_t read_bytes_logits;    /* weight bytes one forward with logits reads */
    size_t read_bytes_no_logits; /* ... without the lm_head */
    size_t kv_bytes_per_pos;     /* 2 * n_layers * n_kv_heads * d_head * (4, or 2 for a bf16 cache)
                                    (this rank's heads) */
    int tp_rank, tp_size;        /* tensor-parallel position of this process */
    int expert_parallel;         /* 1: a MoE model split by experts (attention replicated);
                                    0: one GPU, or rows split (tensor parallelism) */
} mf_model_info;

/* GenStats (include/minfer/base/stats.hpp:3-15) */
typedef struct mf_gen_stats {
    int num_tokens_gen;
    float ttft, throughput, prefill_time, bandwidth;
    double decode_seconds;
    double bytes_read;
} mf_gen_stats;

/* Parse the GGUF file and build the layer list; rank selects the manager
 * rank (device) the model lives on. mf_init must have been called. */
int mf_model_load(const char* gguf_path, const mf_run_params* rp, int rank, mf_model** out);
/* KV cache element type (no reference counterpart: the reference keeps fp32):
 * MF_F32 (default) or, opt-in, MF_BF16, which halves the cache's bytes and
 * rounds every appended K/V row to nearest even (attention still computes in
 * fp32 on the widened values; logits then differ from the reference's by the
 * rounding's effect). Call before mf_model_to_cuda. */
int mf_model_set_kv_dtype(mf_model* m, int dtype);
/* BaseModel::set_device(DeviceType::CUDA): upload weights, allocate RunState. */
int mf_model_to_cuda(mf_model* m);

/* Tensor parallelism (no reference counterpart; the reference runs one
 * device): rank tp_rank of tp_size loads its shard of the GGUF (Q/K/V by
 * KV-head group, O and down by input columns, gate/up by FFN rows, lm_head
 * by vocabulary rows; dense FFN models). After mf_model_to_cuda every rank
 * exports MF_COMM_HANDLE_BYTES with mf_model_comm_handle; the caller
 * exchanges them (e.g. torch.distributed all_gather) and passes all of them,
 * ordered by tp_rank, to mf_model_comm_connect. From then on every rank runs
 * the same calls (forward / generate / decode_chained) with the same tokens;
 * greedy ids and sampled ids come out identical on every rank. */
int mf_model_load_tp(const char* gguf_path, const mf_run_params* rp, int rank, int tp_rank, int tp_size,
                     mf_model** out);
int mf_model_comm_handle(const mf_model* m, void* out, size_t n);
int mf_model_comm_connect(mf_model* m, const void* handles, size_t n);
/* Exchange status bits since the last call (0: every wait succeeded); synchronises. */
int mf_model_comm_status(mf_model* m, int* status);
int mf_model_info_get(const mf_model* m, mf_model_info* out);
void mf_model_free(mf_model* m);

/* BaseModel::forward for one token at `pos` (src/base/model.cpp:36-59).
 * host_logits != 0 copies the logits to host memory (mf_model_logits). */
int mf_model_forward(mf_model* m, uint32_t token, int pos, int compute_logits, int host_logits);
/* Logits of the last forward that computed them with host_logits set. */
int mf_model_logits(const mf_model* m, float* out, size_t n);
/* Greedy id (first maximum) of the last forward that computed logits. */
int mf_model_argmax(const mf_model* m, uint32_t* out);

/* BaseModel::generate without the tokenizer (src/base/model.cpp:99-186):
 * prompt, then sample -> append -> forward. flags: bit0 stop at EOS,
 * bit1 record the top-2 logit margin of every step into margins[n_gen].
 * forced (may be NULL): teacher forcing — the model's pick of step i is
 * reported in out_ids[i] but forced[i] is fed back. Returns the number of
 * generated ids in *n_out. */
int mf_model_generate(mf_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_gen, int flags,
                      const uint32_t* forced, uint32_t* out_ids, size_t* n_out, float* margins,
                      mf_gen_stats* stats);
/* The same, also copying the logits the id of step steps[i] was drawn from
 * (step 0 = the first generated id) into logits_out[i * vocab_size ...] for
 * i < n_steps (the logits are then read back every step). */
int mf_model_generate_logits(mf_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_gen, int flags,
                             const uint32_t* forced, uint32_t* out_ids, size_t* n_out, float* margins,
                             mf_gen_stats* stats, const size_t* steps, size_t n_steps, float* logits_out);
#define MF_GEN_STOP_AT_EOS 1
#define MF_GEN_MARGINS 2
#define MF_GEN_TOKEN_PREFILL 4 /* prefill token by token (the reference's loop) instead of batched */

/* Batched prefill (no reference counterpart; the reference prefills token by
 * token, src/base/model.cpp:120-129): tokens at positions [pos0, pos0 + n)
 * go through every layer as tcgen05 GEMMs, filling the KV cache; with
 * compute_logits the last token's logits / greedy id are then available as
 * after mf_model_forward. Dense models with bf16 weights, or fp32 weights (kept
 * as bf16 hi + lo copies for the GEMMs, two products each), and MoE models
 * with bf16 experts (tokens grouped by expert, grouped GEMMs); f16 weights
 * return MF_E_UNSUPPORTED (use mf_model_forward per token). */
int mf_model_prefill(mf_model* m, const uint32_t* tokens, size_t n, int pos0, int compute_logits, int host_logits);

/* BaseModel::benchmark (src/base/model.cpp:188-236): pp512 (512 random ids
 * from std::mt19937(seed), logits on the last) then tg128 (128 forwards of
 * fresh random ids at positions 0..127); stats as the reference reports them
 * (prefill_time = ttft, throughput = 128 / decode time, bandwidth = bytes the
 * reference counts / total time). flags: MF_GEN_TOKEN_PREFILL runs the 512
 * prompt ids as decode frames, as the reference does; otherwise the batched
 * tensor-core prefill is used when the model supports it. */
int mf_model_benchmark(mf_model* m, int flags, mf_gen_stats* stats);

/* Greedy decode of n tokens with the device feeding itself (no host round
 * trip between tokens), starting with `token` at `start_pos`. Blocks until
 * done; returns the last greedy id. */
int mf_model_decode_chained(mf_model* m, uint32_t token, int start_pos, int n, uint32_t* last_id);

/* Resets the sampler (RNG stream and presence set) to its initial state. */
int mf_model_reset_sampler(mf_model* m);

/* Test access: experts selected at `layer` by the last forward (k ids and
 * weights), the KV rows [0, n_pos) of `layer` in the reference's
 * [pos][kv_head][d_head] order, and the residual stream x. */
int mf_model_experts(const mf_model* m, int layer, int* ids, float* weights);
/* The expert ids / weights ([n_tokens][k] each) the last batched prefill
 * (mf_model_prefill) chose at `layer` for its first n_tokens tokens (MoE
 * models; a prefill of several chunks keeps the last chunk's). */
int mf_model_prefill_experts(const mf_model* m, int layer, int* ids, float* weights, int n_tokens);
int mf_model_kv(const mf_model* m, int layer, float* k, float* v, int n_pos);
int mf_model_x(const mf_model* m, float* x);

/* The host sampler alone (Sampler::sample, src/base/sampler.cpp:34-117): a
 * fresh sampler with rp's settings, the `n_seen` ids of `seen` added for the
 * presence penalty, then `n_draws` draws from the same logits (the RNG
 * advances between draws). No GPU involved. */
int mf_sample(const float* logits, size_t vocab, const mf_run_params* rp, const uint32_t* seen, size_t n_seen,
              size_t n_draws, uint32_t* out);

/* The draw generate() makes when a frame reads back only the device's top-k
 * candidates (mf_topk: the top_k + 1 largest logits, largest first, equal
 * values lower index first): Sampler::sample_candidates on that list, or the
 * whole-vocabulary Sampler::sample when two of those values are equal (their
 * order in the reference's nth_element + sort list is the library's). The
 * candidate list is built here on the host in the device's order; n_draws
 * draws, the RNG advancing between them; no presence penalty. No GPU involved. */
int mf_sample_candidates(const float* logits, size_t vocab, const mf_run_params* rp, size_t n_draws, uint32_t* out);

/* Prompt ids as BaseModel::benchmark draws them (src/base/model.cpp:189-193):
 * std::mt19937(seed) + std::uniform_int_distribution<>(0, vocab-1). */
int mf_random_prompt(int seed, uint32_t vocab, size_t n, uint32_t* out);

/* ---- tokenizer (Qwen3Tokenizer, include/minfer/models/qwen3/tokenizer.hpp;
 * src/models/qwen3/tokenizer.cpp). Host only, no GPU involved. Functions that
 * return bytes or ids write at most `cap` of them and set *n to the full count
 * (call again with a larger buffer when *n > cap). */
typedef struct mf_tokenizer mf_tokenizer;

/* Qwen3Tokenizer::Qwen3Tokenizer (tokenizer.cpp:12-41) from the GGUF keys
 * tokenizer.ggml.{tokens, merges, token_type, eos_token_id,
 * padding_token_id} and tokenizer.chat_template (the keys the reference's
 * tokenizer test reads, tests/src/qwen3/tokenizer/tokenizer.cpp:20-25). */
int mf_tokenizer_load(const char* gguf_path, mf_tokenizer** out);
/* The same from arrays: tokens[i] has token_lens[i] bytes (byte form), merges
 * are "left right" byte strings. MF_E_INVALID for mismatched lengths or a
 * merge without a space (tokenizer.cpp:28-30,124-128). */
int mf_tokenizer_create(const char* const* tokens, const size_t* token_lens, const uint32_t* token_types,
                        size_t n_tokens, const char* const* merges, const size_t* merge_lens, size_t n_merges,
                        const char* chat_template, uint32_t eos_id, uint32_t pad_id, mf_tokenizer** out);
void mf_tokenizer_free(mf_tokenizer* t);
int mf_tokenizer_info(const mf_tokenizer* t, size_t* vocab_size, uint32_t* eos_id, uint32_t* pad_id);
/* encode (tokenizer.cpp:45-62). MF_E_INVALID when the vocabulary lacks a byte
 * or merged string the text needs (the reference throws there). */
int mf_tokenizer_encode(const mf_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap, size_t* n);
/* decode (tokenizer.cpp:76-87): unused tokens decode as "<UNK>";
 * MF_E_INVALID for an id past the vocabulary. */
int mf_tokenizer_decode(const mf_tokenizer* t, const uint32_t* ids, size_t n_ids, char* out, size_t cap, size_t* n);
/* The pieces encode splits the text into (regex_split, tokenizer.cpp:176-226):
 * ends[i] = byte offset one past piece i. */
int mf_tokenizer_pre_split(const mf_tokenizer* t, const char* text, size_t len, size_t* ends, size_t cap, size_t* n);
/* apply_chat_template (tokenizer.cpp:291-335): messages_json is a JSON array
 * of {"role", "content", "reasoning_content"?, "tool_calls"?: [{"name",
 * "arguments"}]}, tools_json a JSON array of {"name", "description",
 * "parameters"} (or NULL for none), the objects the reference builds from its
 * Message/Tool structs (any JSON messages are accepted, e.g. OpenAI-shaped
 * tool calls). MF_E_STATE for errors the template raises, MF_E_UNSUPPORTED
 * for template constructs not built (recursive loops, call blocks). */
int mf_tokenizer_apply_chat_template(const mf_tokenizer* t, const char* messages_json, const char* tools_json,
                                     int add_generation_prompt, char* out, size_t cap, size_t* n);

#ifdef __cplusplus
}
#endif
#endif /* MINFER_MODEL_H */
