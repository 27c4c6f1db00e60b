// Host runtime structures: model weights, workspace, KV cache.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/qwen3_b200.h"
#include "kernels.h"

namespace qw {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define QW_CUDA(expr)                                                                              \
    do {                                                                                           \
        cudaError_t _e = (expr);                                                                   \
        if (_e != cudaSuccess)                                                                     \
            throw ::qw::Error(QW_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e));     \
    } while (0)

// Hyperparameters used by the path (crates/base-mlx-core/src/model/config.rs:11-201).
struct Config {
    std::string model_type;
    int hidden = 0, intermediate = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
    float eps = 1e-6f, rope_theta = 10000.f;
    int max_pos_emb = 4096;
    bool tied = false;
    int bits = 0, group_size = 0;
    bool quantized = false;
    int bos = -1;
    std::vector<int> eos;
};
Config parse_config(const std::string& json_text);

// One quantized linear on the device (this rank's shard).
struct QLin {
    uint32_t* w = nullptr;
    bf16* s = nullptr;
    bf16* b = nullptr;
    int n = 0, k = 0;
};

struct Layer {
    bf16 *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    QLin q, k, v, o, gate, up, down;
};

struct TensorRef {  // for export
    void* ptr;
    size_t bytes;
};

struct Workspace {
    int cap_rows = 0;     // activation rows available
    int cap_logits = 0;   // logits rows available
    bf16 *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *attn = nullptr,
         *mlp = nullptr, *logits = nullptr;
    float* f32 = nullptr;        // tensor-parallel partial sums [rows, hidden]
    void* xh = nullptr;          // fp16 activations for the tcgen05 prefill GEMM
    size_t xh_bytes = 0;
    int* ids = nullptr;          // input token ids [rows]
    int* argmax = nullptr;       // [rows]
    unsigned long long* amax_partial = nullptr;  // lm_head per-CTA maxima [row blocks, rows]
    unsigned long long* amax_keys = nullptr;  // [logits rows] (tensor-parallel argmax)
    float* attn_part = nullptr;
    unsigned* attn_counters = nullptr;
    int* next_tok = nullptr;     // device-resident greedy loop: next input token
    int* out = nullptr;          // generated tokens
    int out_cap = 0;
    StepCtl* ctl = nullptr;
    BatchCtl* bctl = nullptr;
    float* probs = nullptr;      // sampling: softmax probabilities [vocab]
    SampleCfg* scfg = nullptr;   // sampling parameters of the running generation
    void* sctrl = nullptr;       // sampling control block (zeroed at allocation)
    int generation = 0;          // bumped on reallocation (invalidates graphs)
    std::vector<void*> allocs;
};

struct TpComm;  // tensor-parallel communicator (NCCL), defined in tp.cu
struct TpPeer;  // peer-memory exchange block for the decode reductions, defined in tp.cu
struct MkState;  // persistent decode kernel: packed weights + sync words, defined in decode_mk.cu

}  // namespace qw

struct qw_cache;

struct qw_model {
    qw::Config cfg;
    int device = 0;
    int tp_rank = 0, tp_size = 1;
    int hq_l = 0, hkv_l = 0, inter_l = 0, vocab_l = 0;  // this rank's shard sizes
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    qw::QLin embed;
    qw::QLin lm_head;  // == embed when tied (shares memory)
    std::vector<qw::Layer> layers;
    bf16* final_norm = nullptr;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    int rope_max_pos = 0;
    int* d_err = nullptr;
    std::map<std::string, qw::TensorRef> tensors;
    qw::Workspace ws;
    qw::TpComm* tp = nullptr;
    qw::TpPeer* tpp = nullptr;
    std::vector<qw_cache*> caches;  // live caches (freed with the model)
    qw_cache* gen_cache = nullptr;  // cache used by the generate entry points
    void* spec_state = nullptr;     // speculative-decoding graphs (spec.cu)
    qw::MkState* mk = nullptr;      // persistent decode kernel state (decode_mk.cu)
    // diagnostics (qw_forward_trace): when set, a forward copies the residual
    // stream [S, hidden] after the embedding and after every layer into
    // trace[0..layers] (bf16, [layers + 1][S][hidden]), the residual after
    // each layer's attention block into trace_mid ([layers][S][hidden]) and
    // the attention output (o_proj input) into trace_attn ([layers][S][heads * 128])
    bf16* trace = nullptr;
    bf16* trace_mid = nullptr;
    bf16* trace_attn = nullptr;
    ~qw_model();
};

struct qw_cache {
    qw_model* m = nullptr;
    int max_pos = 0;
    bf16* k = nullptr;  // [layers, kv_heads_local, max_pos, 128]
    bf16* v = nullptr;
    int* d_seq_len = nullptr;
    int seq_len = 0;  // host mirror
    // captured decode-step graph (greedy device loop)
    cudaGraphExec_t step_graph = nullptr;
    int step_graph_gen = -1;
    // captured decode-step graph of the sampled device loop
    cudaGraphExec_t sample_graph = nullptr;
    int sample_graph_gen = -1;
    ~qw_cache();
    bf16* kl(int layer) const;
    bf16* vl(int layer) const;
};

namespace qw {

// model.cu
qw_model* model_create(const Config& cfg, int device, int tp_rank, int tp_size);
void model_alloc_weights(qw_model* m);
void model_load_dir(qw_model* m, const std::string& dir);
void model_init_random(qw_model* m, uint64_t seed, int norm_mode);
void ensure_workspace(qw_model* m, int rows, int logits_rows);
void set_cache_len(qw_cache* c, int len);
void check_device_err(qw_model* m);
qw_cache* cache_create(qw_model* m, int max_pos);
qw_cache* cache_for_generate(qw_model* m, int need_pos);

// decode_mk.cu: persistent decode step (S <= 8 rows, one GPU)
void mk_prepare(qw_model* m);
void mk_free(qw_model* m);
// QW_MK_PROFILE diagnostics: copy the persistent kernel's stamp buffer; bytes copied (0 when absent)
size_t mk_prof_read(const qw_model* m, void* dst, size_t bytes);
// A batched step: nseq independent sequences, one new token each (row b of
// the ids / logits / argmax is sequence b, with cache caches[b]).
struct MkBatch {
    qw_cache* const* caches;
    int nseq;
    BatchCtl* bctl;  // device loop bookkeeping, or null
    int b0 = 0;       // first sequence of this launch within the whole batch
    int btotal = 0;   // sequences in the whole batch (0: nseq)
    bool finalize = true;  // this launch completes the step
};
// Largest number of sequences one batched step carries on this model (shared
// memory holds every row's staged activations), 0 without the persistent kernel.
int mk_batch_rows(qw_model* m);
// false when the step does not fit the persistent kernel (the caller runs the kernel chain)
bool mk_forward(qw_model* m, qw_cache* c, const int* d_ids, int S, int logits_mode, bool store_logits,
                int* d_argmax, cudaStream_t st, StepCtl* ctl, int* next_tok, int* out, const int* gate,
                const MkBatch* batch = nullptr);

// forward.cu
// logits_mode: 0 = none, 1 = last row, 2 = all rows
void forward_dev(qw_model* m, qw_cache* c, const int* d_ids, int S, int logits_mode, bool store_logits,
                 int* d_argmax, cudaStream_t st, StepCtl* ctl, int* next_tok, int* out, const int* gate = nullptr);
void generate_greedy_dev(qw_model* m, qw_cache* c, int n_prompt, int max_new, const std::vector<int>& eos,
                         qw_gen_stats* stats, cudaStream_t st);
// nseq prompts decoded together (one persistent step per token for all of them)
void generate_greedy_batch_dev(qw_model* m, qw_cache* const* caches, int nseq, const std::vector<std::vector<int>>& prompts,
                               int max_new, const std::vector<int>& eos, std::vector<std::vector<int>>& outs,
                               qw_gen_stats* stats, cudaStream_t st);
void generate_sampled_dev(qw_model* m, qw_cache* c, int n_prompt, int max_new, const std::vector<int>& eos,
                          const SampleCfg& cfg, qw_gen_stats* stats, cudaStream_t st);

// spec.cu
struct SpecRequest {
    const int* prompt;  // host
    int n_prompt, max_new, k;
    float force_p;
    uint64_t seed;
    const int* forced;  // host, may be null
    int n_forced;
    std::vector<int> eos_target, eos_draft;
    // temperature > 0: speculative sampling (draft tokens drawn from the draft's
    // top-p distribution, accepted with probability min(1, P_target / P_draft),
    // residual draw on rejection); force_p is ignored then
    float temperature = 0.f;
    float top_p = 1.f;
};
void spec_state_free(void* p);
void spec_generate_dev(qw_model* target, qw_model* draft, const SpecRequest& r, std::vector<int>& out,
                       qw_spec_stats* stats);

// tp.cu
void tp_unique_id(void* out, size_t bytes);
void tp_attach(qw_model* m, const void* unique_id, int rank, int size);
void tp_allreduce_sum_f32(qw_model* m, float* buf, size_t count, cudaStream_t st);
void tp_allreduce_max_u64(qw_model* m, unsigned long long* buf, size_t count, cudaStream_t st);
void tp_destroy(qw_model* m);
// peer-memory reductions (decode): this rank's IPC handle, the ranks' handles
// opened, whether the push path is on, GEMV arguments, the reducing kernel
void tp_push_handle(qw_model* m, void* out, size_t bytes);
void tp_push_open(qw_model* m, const void* handles, size_t bytes);
bool tp_push_ready(const qw_model* m);
void tp_push_args(qw_model* m, TpPush& a);
cudaError_t launch_tp_push_reduce(qw_model* m, bf16* x, int S, cudaStream_t st);

}  // namespace qw
