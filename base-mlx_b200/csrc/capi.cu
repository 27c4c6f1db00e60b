// extern "C" boundary (include/qwen3_b200.h).  Each entry point converts
// exceptions into a status code plus a thread-local message, mirroring the
// Result<T, Error> convention of crates/base-mlx-core/src/error.rs:6-32.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "model.h"

namespace {

thread_local std::string g_err;

template <typename F>
int guard(F&& f) {
    try {
        f();
        return QW_OK;
    } catch (const qw::Error& e) {
        g_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_err = e.what();
        return QW_ERR_INFERENCE;
    } catch (...) {
        g_err = "unknown error";
        return QW_ERR_INFERENCE;
    }
}

void need(bool ok, const char* what) {
    if (!ok) throw qw::Error(QW_ERR_INVALID_ARG, what);
}

// engine.rs:266-272: the config's eos ids, else Qwen's 151645 / 151643.
std::vector<int> eos_list(const qw_model* m, const uint32_t* eos, int n_eos) {
    std::vector<int> v;
    if (eos && n_eos > 0) {
        for (int i = 0; i < n_eos; ++i) v.push_back((int)eos[i]);
    } else if (!m->cfg.eos.empty()) {
        v = m->cfg.eos;
    } else {
        v = {151645, 151643};
    }
    return v;
}

void check_ids(const qw_model* m, const uint32_t* ids, int n) {
    for (int i = 0; i < n; ++i)
        if (ids[i] >= (uint32_t)m->cfg.vocab)
            throw qw::Error(QW_ERR_INVALID_ARG, "token id " + std::to_string(ids[i]) + " out of range");
}

}  // namespace

extern "C" {

int qw_last_error(char* buf, size_t len) {
    if (!buf || len == 0) return QW_ERR_INVALID_ARG;
    std::snprintf(buf, len, "%s", g_err.c_str());
    return QW_OK;
}

int qw_version(char* buf, size_t len) {
    return guard([&] {
        need(buf && len, "buf");
        int rt = 0;
        cudaRuntimeGetVersion(&rt);
        std::snprintf(buf, len, "qwen3_b200 sm_100a cudart %d.%d", rt / 1000, (rt % 1000) / 10);
    });
}

int qw_model_load(const char* dir, int device, int tp_rank, int tp_size, qw_model** out) {
    return guard([&] {
        need(dir && out, "dir/out");
        *out = nullptr;
        std::ifstream f(std::string(dir) + "/config.json");
        if (!f) throw qw::Error(QW_ERR_MODEL_LOAD, std::string("missing config.json in ") + dir);
        std::stringstream ss;
        ss << f.rdbuf();
        qw::Config cfg = qw::parse_config(ss.str());
        qw_model* m = qw::model_create(cfg, device, tp_rank, tp_size);
        try {
            qw::model_load_dir(m, dir);
            qw::mk_prepare(m);
        } catch (...) {
            delete m;
            throw;
        }
        *out = m;
    });
}

int qw_model_init_random(const char* config_json, uint64_t seed, int norm_mode, int device, int tp_rank,
                         int tp_size, qw_model** out) {
    return guard([&] {
        need(config_json && out, "config/out");
        *out = nullptr;
        qw::Config cfg = qw::parse_config(config_json);
        qw_model* m = qw::model_create(cfg, device, tp_rank, tp_size);
        try {
            qw::model_init_random(m, seed, norm_mode);
            qw::mk_prepare(m);
        } catch (...) {
            delete m;
            throw;
        }
        *out = m;
    });
}

int qw_model_free(qw_model* m) {
    return guard([&] {
        if (!m) return;
        delete m;  // also frees every cache still attached to the model
    });
}

int qw_model_info_get(const qw_model* m, qw_model_info* o) {
    return guard([&] {
        need(m && o, "model/out");
        const qw::Config& c = m->cfg;
        o->num_layers = c.layers;
        o->hidden = c.hidden;
        o->intermediate = c.intermediate;
        o->num_heads = c.heads;
        o->num_kv_heads = c.kv_heads;
        o->head_dim = c.head_dim;
        o->vocab = c.vocab;
        o->tied_embeddings = c.tied ? 1 : 0;
        o->tp_rank = m->tp_rank;
        o->tp_size = m->tp_size;
        o->rms_eps = c.eps;
        o->rope_theta = c.rope_theta;
        o->weight_bytes = m->arena_bytes;
    });
}

int qw_model_export_tensor(const qw_model* m, const char* name, void* dst, size_t bytes) {
    return guard([&] {
        need(m && name && dst, "model/name/dst");
        auto it = m->tensors.find(name);
        if (it == m->tensors.end()) throw qw::Error(QW_ERR_INVALID_ARG, std::string("no tensor named ") + name);
        if (it->second.bytes != bytes)
            throw qw::Error(QW_ERR_INVALID_ARG, "size mismatch: tensor has " + std::to_string(it->second.bytes) + " bytes");
        QW_CUDA(cudaSetDevice(m->device));
        QW_CUDA(cudaMemcpy(dst, it->second.ptr, bytes, cudaMemcpyDeviceToHost));
    });
}

int qw_model_stream(const qw_model* m, void** s) {
    return guard([&] {
        need(m && s, "model/out");
        *s = (void*)m->stream;
    });
}

int qw_tp_unique_id(void* out, size_t bytes) {
    return guard([&] {
        need(out, "out");
        qw::tp_unique_id(out, bytes);
    });
}

int qw_model_tp_attach(qw_model* m, const void* uid, int rank, int size) {
    return guard([&] {
        need(m && uid, "model/id");
        qw::tp_attach(m, uid, rank, size);
    });
}

int qw_tp_exchange_handle(qw_model* m, void* out, size_t bytes) {
    return guard([&] {
        need(m && out, "model/out");
        qw::tp_push_handle(m, out, bytes);
    });
}

int qw_tp_exchange_open(qw_model* m, const void* handles, size_t bytes) {
    return guard([&] {
        need(m && handles, "model/handles");
        qw::tp_push_open(m, handles, bytes);
    });
}

// speculative.rs:40-54
int qw_check_compatible(const qw_model* t, const qw_model* d) {
    return guard([&] {
        need(t && d, "models");
        if (t->cfg.vocab != d->cfg.vocab)
            throw qw::Error(QW_ERR_MODEL_LOAD, "draft/target vocab mismatch: target=" + std::to_string(t->cfg.vocab) +
                                                  " draft=" + std::to_string(d->cfg.vocab));
        if (t->cfg.model_type != d->cfg.model_type)
            throw qw::Error(QW_ERR_MODEL_LOAD, "draft/target architecture mismatch: target=" + t->cfg.model_type +
                                                  " draft=" + d->cfg.model_type);
    });
}

int qw_cache_new(qw_model* m, int max_pos, qw_cache** out) {
    return guard([&] {
        need(m && out, "model/out");
        *out = qw::cache_create(m, max_pos);
    });
}

int qw_cache_free(qw_cache* c) {
    return guard([&] {
        if (!c) return;
        qw_model* m = c->m;
        if (m) {
            cudaSetDevice(m->device);
            cudaStreamSynchronize(m->stream);
            for (auto it = m->caches.begin(); it != m->caches.end(); ++it)
                if (*it == c) {
                    m->caches.erase(it);
                    break;
                }
            if (m->gen_cache == c) m->gen_cache = nullptr;
        }
        delete c;
    });
}

int qw_cache_reset(qw_cache* c) {
    return guard([&] {
        need(c, "cache");
        qw::set_cache_len(c, 0);
    });
}

int qw_cache_truncate(qw_cache* c, int new_len) {
    return guard([&] {
        need(c, "cache");
        need(new_len >= 0, "new_len");
        if (new_len < c->seq_len) qw::set_cache_len(c, new_len);
    });
}

int qw_cache_len(const qw_cache* c, int* out) {
    return guard([&] {
        need(c && out, "cache/out");
        *out = c->seq_len;
    });
}

int qw_kv_slice_update(qw_cache* c, int layer, int which_v, const uint16_t* upd, int start, int stop) {
    return guard([&] {
        need(c && upd, "cache/update");
        qw_model* m = c->m;
        need(layer >= 0 && layer < m->cfg.layers, "layer");
        need(start >= 0 && stop > start && stop <= c->max_pos, "start/stop");
        const size_t D = m->cfg.head_dim, n = (size_t)(stop - start);
        bf16* base = (which_v ? c->vl(layer) : c->kl(layer)) + (size_t)start * D;
        QW_CUDA(cudaSetDevice(m->device));
        QW_CUDA(cudaMemcpy2DAsync(base, (size_t)c->max_pos * D * 2, upd, n * D * 2, n * D * 2, (size_t)m->hkv_l,
                                  cudaMemcpyHostToDevice, m->stream));
        QW_CUDA(cudaStreamSynchronize(m->stream));
    });
}

int qw_kv_read(const qw_cache* c, int layer, int which_v, uint16_t* dst, int start, int stop) {
    return guard([&] {
        need(c && dst, "cache/dst");
        qw_model* m = c->m;
        need(layer >= 0 && layer < m->cfg.layers, "layer");
        need(start >= 0 && stop > start && stop <= c->max_pos, "start/stop");
        const size_t D = m->cfg.head_dim, n = (size_t)(stop - start);
        const bf16* base = (which_v ? c->vl(layer) : c->kl(layer)) + (size_t)start * D;
        QW_CUDA(cudaSetDevice(m->device));
        QW_CUDA(cudaMemcpy2DAsync(dst, n * D * 2, base, (size_t)c->max_pos * D * 2, n * D * 2, (size_t)m->hkv_l,
                                  cudaMemcpyDeviceToHost, m->stream));
        QW_CUDA(cudaStreamSynchronize(m->stream));
    });
}

int qw_forward(qw_model* m, qw_cache* c, const uint32_t* ids, int n, int all_rows, uint16_t* logits_out,
               uint32_t* argmax_out) {
    return guard([&] {
        need(m && c && ids, "model/cache/ids");
        need(c->m == m, "cache belongs to another model");
        need(n >= 1, "n must be >= 1");
        // qwen3.rs:423-428
        if (c->seq_len + n > c->max_pos)
            throw qw::Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(c->seq_len + n) +
                                                     " positions, max " + std::to_string(c->max_pos));
        check_ids(m, ids, n);
        QW_CUDA(cudaSetDevice(m->device));
        const int rows = all_rows ? n : 1;
        qw::ensure_workspace(m, n, rows);
        std::vector<int> h(ids, ids + n);
        cudaStream_t st = m->stream;
        QW_CUDA(cudaMemcpyAsync(m->ws.ids, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
        qw::forward_dev(m, c, m->ws.ids, n, all_rows ? 2 : 1, logits_out != nullptr, m->ws.argmax, st, nullptr,
                        nullptr, nullptr);
        if (logits_out)
            QW_CUDA(cudaMemcpyAsync(logits_out, m->ws.logits, (size_t)rows * m->vocab_l * 2, cudaMemcpyDeviceToHost, st));
        std::vector<int> am(rows);
        QW_CUDA(cudaMemcpyAsync(am.data(), m->ws.argmax, (size_t)rows * 4, cudaMemcpyDeviceToHost, st));
        QW_CUDA(cudaStreamSynchronize(st));
        c->seq_len += n;
        qw::check_device_err(m);
        if (argmax_out)
            for (int i = 0; i < rows; ++i) argmax_out[i] = (uint32_t)am[i];
    });
}

int qw_forward_trace(qw_model* m, qw_cache* c, const uint32_t* ids, int n, uint16_t* residual_out,
                     uint16_t* mid_out, uint16_t* attn_out, uint16_t* logits_out, uint32_t* argmax_out) {
    return guard([&] {
        need(m && c && ids && residual_out, "model/cache/ids/residual_out");
        need(c->m == m, "cache belongs to another model");
        need(n >= 1, "n must be >= 1");
        if (c->seq_len + n > c->max_pos)
            throw qw::Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(c->seq_len + n) +
                                                     " positions, max " + std::to_string(c->max_pos));
        check_ids(m, ids, n);
        QW_CUDA(cudaSetDevice(m->device));
        qw::ensure_workspace(m, n, 1);
        const int L = m->cfg.layers, H = m->cfg.hidden, QD = m->hq_l * m->cfg.head_dim;
        const size_t tr_bytes = (size_t)(L + 1) * n * H * 2, mid_bytes = (size_t)L * n * H * 2,
                     attn_bytes = (size_t)L * n * QD * 2;
        bf16* tr = nullptr;
        QW_CUDA(cudaMalloc(&tr, tr_bytes + mid_bytes + attn_bytes));
        struct Release {
            qw_model* m;
            bf16* p;
            ~Release() {
                m->trace = m->trace_mid = m->trace_attn = nullptr;
                cudaFree(p);
            }
        } rel{m, tr};
        m->trace = tr;
        m->trace_mid = tr + tr_bytes / 2;
        m->trace_attn = m->trace_mid + mid_bytes / 2;
        std::vector<int> h(ids, ids + n);
        cudaStream_t st = m->stream;
        QW_CUDA(cudaMemcpyAsync(m->ws.ids, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
        qw::forward_dev(m, c, m->ws.ids, n, 1, logits_out != nullptr, m->ws.argmax, st, nullptr, nullptr, nullptr);
        QW_CUDA(cudaMemcpyAsync(residual_out, tr, tr_bytes, cudaMemcpyDeviceToHost, st));
        if (mid_out) QW_CUDA(cudaMemcpyAsync(mid_out, m->trace_mid, mid_bytes, cudaMemcpyDeviceToHost, st));
        if (attn_out) QW_CUDA(cudaMemcpyAsync(attn_out, m->trace_attn, attn_bytes, cudaMemcpyDeviceToHost, st));
        if (logits_out)
            QW_CUDA(cudaMemcpyAsync(logits_out, m->ws.logits, (size_t)m->vocab_l * 2, cudaMemcpyDeviceToHost, st));
        int am = 0;
        QW_CUDA(cudaMemcpyAsync(&am, m->ws.argmax, 4, cudaMemcpyDeviceToHost, st));
        QW_CUDA(cudaStreamSynchronize(st));
        c->seq_len += n;
        qw::check_device_err(m);
        if (argmax_out) *argmax_out = (uint32_t)am;
    });
}

int qw_debug_decode_stamps(const qw_model* m, void* dst_host, size_t bytes, size_t* written) {
    return guard([&] {
        need(m && dst_host && written, "model/dst/written");
        QW_CUDA(cudaSetDevice(m->device));
        *written = qw::mk_prof_read(m, dst_host, bytes);
    });
}

int qw_generate_greedy(qw_model* m, const uint32_t* prompt, int n_prompt, int max_new, const uint32_t* eos,
                       int n_eos, uint32_t* out, int* n_out, qw_gen_stats* stats) {
    return guard([&] {
        need(m && prompt && out && n_out, "model/prompt/out");
        need(n_prompt >= 1, "empty prompt");
        check_ids(m, prompt, n_prompt);
        // the reference loop always picks at least one token (engine.rs:161-173)
        const int mn = std::max(max_new, 1);
        QW_CUDA(cudaSetDevice(m->device));
        qw_cache* c = qw::cache_for_generate(m, n_prompt + mn);
        qw::ensure_workspace(m, n_prompt, 8);
        cudaStream_t st = m->stream;
        std::vector<int> h(prompt, prompt + n_prompt);
        QW_CUDA(cudaMemcpyAsync(m->ws.ids, h.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st));
        qw_gen_stats s;
        std::memset(&s, 0, sizeof(s));
        qw::generate_greedy_dev(m, c, n_prompt, mn, eos_list(m, eos, n_eos), &s, st);
        const int cnt = std::min(s.completion_tokens, mn);
        const int written = cnt - (s.finish_reason == 1 ? 1 : 0);
        std::vector<int> o((size_t)std::max(written, 1));
        if (written > 0) QW_CUDA(cudaMemcpy(o.data(), m->ws.out, (size_t)written * 4, cudaMemcpyDeviceToHost));
        for (int i = 0; i < written; ++i) out[i] = (uint32_t)o[i];
        *n_out = written;
        if (stats) *stats = s;
        qw::set_cache_len(c, 0);  // cache.reset() at the end of a request (engine.rs:183)
        qw::check_device_err(m);
    });
}

int qw_forward_batch(qw_model* m, qw_cache* const* caches, int nseq, const uint32_t* ids, uint16_t* logits_out,
                     uint32_t* argmax_out) {
    return guard([&] {
        need(m && caches && ids, "model/caches/ids");
        need(nseq >= 1 && nseq <= 8, "nseq must be 1..8");
        need(m->tp_size == 1, "batched decode runs on one GPU (tp_size 1)");
        for (int b = 0; b < nseq; ++b) {
            need(caches[b] != nullptr, "null cache");
            need(caches[b]->m == m, "cache belongs to another model");
            for (int b2 = 0; b2 < b; ++b2) need(caches[b2] != caches[b], "a cache appears twice in the batch");
            if (caches[b]->seq_len + 1 > caches[b]->max_pos)
                throw qw::Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " +
                                                         std::to_string(caches[b]->seq_len + 1) + " positions, max " +
                                                         std::to_string(caches[b]->max_pos));
        }
        check_ids(m, ids, nseq);
        QW_CUDA(cudaSetDevice(m->device));
        qw::ensure_workspace(m, nseq, nseq);
        std::vector<int> h(ids, ids + nseq);
        cudaStream_t st = m->stream;
        QW_CUDA(cudaMemcpyAsync(m->ws.ids, h.data(), (size_t)nseq * 4, cudaMemcpyHostToDevice, st));
        // sub-batches of at most mk_batch_rows sequences, sizes balanced
        const int cap = qw::mk_batch_rows(m);
        if (cap < 1) throw qw::Error(QW_ERR_UNSUPPORTED, "this model does not fit the batched decode step");
        const int nch = (nseq + cap - 1) / cap;
        std::vector<int> am(nseq);
        for (int ci = 0, b0 = 0; ci < nch; ++ci) {
            const int nc = nseq / nch + (ci < nseq % nch ? 1 : 0);
            qw::MkBatch mb{caches + b0, nc, nullptr, b0, nseq, ci == nch - 1};
            if (!qw::mk_forward(m, caches[b0], m->ws.ids + b0, nc, 2, logits_out != nullptr, m->ws.argmax, st,
                                nullptr, nullptr, nullptr, nullptr, &mb))
                throw qw::Error(QW_ERR_UNSUPPORTED, "this model / batch does not fit the batched decode step");
            if (logits_out)
                QW_CUDA(cudaMemcpyAsync(logits_out + (size_t)b0 * m->vocab_l, m->ws.logits,
                                        (size_t)nc * m->vocab_l * 2, cudaMemcpyDeviceToHost, st));
            QW_CUDA(cudaMemcpyAsync(am.data() + b0, m->ws.argmax, (size_t)nc * 4, cudaMemcpyDeviceToHost, st));
            b0 += nc;
        }
        QW_CUDA(cudaStreamSynchronize(st));
        for (int b = 0; b < nseq; ++b) caches[b]->seq_len += 1;
        qw::check_device_err(m);
        if (argmax_out)
            for (int b = 0; b < nseq; ++b) argmax_out[b] = (uint32_t)am[b];
    });
}

int qw_generate_greedy_batch(qw_model* m, qw_cache* const* caches, int nseq, const uint32_t* prompts,
                             const int* n_prompt, int max_new, const uint32_t* eos, int n_eos, uint32_t* out,
                             int* n_out, qw_gen_stats* stats) {
    return guard([&] {
        need(m && caches && prompts && n_prompt && out && n_out, "model/caches/prompts/out");
        need(nseq >= 1 && nseq <= 8, "nseq must be 1..8");
        need(m->tp_size == 1, "batched decode runs on one GPU (tp_size 1)");
        const int mn = std::max(max_new, 1);
        std::vector<std::vector<int>> pr(nseq);
        size_t off = 0;
        int longest = 0;
        for (int b = 0; b < nseq; ++b) {
            need(caches[b] != nullptr && caches[b]->m == m, "cache missing or of another model");
            need(n_prompt[b] >= 1, "empty prompt");
            check_ids(m, prompts + off, n_prompt[b]);
            pr[b].assign(prompts + off, prompts + off + n_prompt[b]);
            off += (size_t)n_prompt[b];
            longest = std::max(longest, n_prompt[b]);
        }
        QW_CUDA(cudaSetDevice(m->device));
        qw::ensure_workspace(m, longest, 8);
        std::vector<std::vector<int>> outs;
        qw_gen_stats s;
        std::memset(&s, 0, sizeof(s));
        qw::generate_greedy_batch_dev(m, caches, nseq, pr, mn, eos_list(m, eos, n_eos), outs, &s, m->stream);
        for (int b = 0; b < nseq; ++b) {
            n_out[b] = (int)outs[b].size();
            for (size_t i = 0; i < outs[b].size(); ++i) out[(size_t)b * mn + i] = (uint32_t)outs[b][i];
        }
        if (stats) *stats = s;
        qw::check_device_err(m);
    });
}

int qw_generate_sampled(qw_model* m, const uint32_t* prompt, int n_prompt, int max_new, float temperature,
                        float top_p, uint64_t seed, int same_draw, const uint32_t* eos, int n_eos, uint32_t* out,
                        int* n_out, qw_gen_stats* stats) {
    if (!(temperature > 0.f))  // engine.rs:197: greedy when temperature <= 0
        return qw_generate_greedy(m, prompt, n_prompt, max_new, eos, n_eos, out, n_out, stats);
    return guard([&] {
        need(m && prompt && out && n_out, "model/prompt/out");
        need(n_prompt >= 1, "empty prompt");
        need(top_p == top_p, "top_p is NaN");
        check_ids(m, prompt, n_prompt);
        const int mn = std::max(max_new, 1);
        QW_CUDA(cudaSetDevice(m->device));
        qw_cache* c = qw::cache_for_generate(m, n_prompt + mn);
        qw::ensure_workspace(m, n_prompt, 8);
        cudaStream_t st = m->stream;
        std::vector<int> h(prompt, prompt + n_prompt);
        QW_CUDA(cudaMemcpyAsync(m->ws.ids, h.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st));
        qw::SampleCfg cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.temperature = temperature;
        cfg.top_p = top_p;
        cfg.seed = seed;
        cfg.same_draw = same_draw ? 1 : 0;
        qw_gen_stats s;
        std::memset(&s, 0, sizeof(s));
        qw::generate_sampled_dev(m, c, n_prompt, mn, eos_list(m, eos, n_eos), cfg, &s, st);
        const int cnt = std::min(s.completion_tokens, mn);
        const int written = cnt - (s.finish_reason == 1 ? 1 : 0);
        std::vector<int> o((size_t)std::max(written, 1));
        if (written > 0) QW_CUDA(cudaMemcpy(o.data(), m->ws.out, (size_t)written * 4, cudaMemcpyDeviceToHost));
        for (int i = 0; i < written; ++i) out[i] = (uint32_t)o[i];
        *n_out = written;
        if (stats) *stats = s;
        qw::set_cache_len(c, 0);
        qw::check_device_err(m);
    });
}

int qw_sample_topp(const void* logits, int vocab, float temperature, float top_p, uint64_t seed, uint64_t counter,
                   void* scratch, int32_t* token_out, void* stream) {
    return guard([&] {
        need(logits && scratch && token_out, "logits/scratch/token_out");
        need(vocab >= 1, "vocab must be positive");
        need(top_p == top_p && temperature == temperature, "NaN parameter");
        qw::SampleArgs a;
        std::memset(&a, 0, sizeof(a));
        a.logits = (const bf16*)logits;
        a.V = vocab;
        a.cfg.temperature = temperature;
        a.cfg.top_p = top_p;
        a.cfg.seed = seed;
        a.ctrl = scratch;
        a.probs = (float*)((char*)scratch + qw::QW_SAMPLE_CTRL_BYTES);
        a.counter = counter;
        a.token_out = token_out;
        QW_CUDA(qw::launch_sample(a, (cudaStream_t)stream));
    });
}

int qw_spec_generate(qw_model* target, qw_model* draft, const uint32_t* prompt, int n_prompt, int max_new, int k,
                     float force_p, uint64_t seed, const uint32_t* forced, int n_forced, const uint32_t* eos,
                     int n_eos, uint32_t* out, int* n_out, qw_spec_stats* stats) {
    return guard([&] {
        need(target && draft && prompt && out && n_out, "target/draft/prompt/out");
        need(n_prompt >= 1, "empty prompt");
        need(n_forced >= 0, "n_forced");
        if (qw_check_compatible(target, draft) != QW_OK) throw qw::Error(QW_ERR_MODEL_LOAD, g_err);
        check_ids(target, prompt, n_prompt);
        if (forced) check_ids(target, forced, n_forced);
        QW_CUDA(cudaSetDevice(target->device));
        std::vector<int> p(prompt, prompt + n_prompt);
        std::vector<int> f;
        if (forced) f.assign(forced, forced + n_forced);
        qw::SpecRequest r;
        r.prompt = p.data();
        r.n_prompt = n_prompt;
        r.max_new = max_new;
        r.k = k;
        r.force_p = force_p;
        r.seed = seed;
        r.forced = forced ? f.data() : nullptr;
        r.n_forced = forced ? n_forced : 0;
        r.eos_target = eos_list(target, eos, n_eos);
        r.eos_draft = eos_list(draft, eos, n_eos);
        std::vector<int> toks;
        qw_spec_stats s;
        std::memset(&s, 0, sizeof(s));
        qw::spec_generate_dev(target, draft, r, toks, &s);
        for (size_t i = 0; i < toks.size(); ++i) out[i] = (uint32_t)toks[i];
        *n_out = (int)toks.size();
        if (stats) *stats = s;
    });
}

int qw_spec_generate_sampled(qw_model* target, qw_model* draft, const uint32_t* prompt, int n_prompt, int max_new,
                             int k, float temperature, float top_p, uint64_t seed, const uint32_t* eos, int n_eos,
                             uint32_t* out, int* n_out, qw_spec_stats* stats) {
    if (!(temperature > 0.f))  // greedy: the exact greedy loop
        return qw_spec_generate(target, draft, prompt, n_prompt, max_new, k, 0.f, seed, nullptr, 0, eos, n_eos, out,
                                n_out, stats);
    return guard([&] {
        need(target && draft && prompt && out && n_out, "target/draft/prompt/out");
        need(n_prompt >= 1, "empty prompt");
        need(top_p == top_p && temperature == temperature, "NaN parameter");
        if (qw_check_compatible(target, draft) != QW_OK) throw qw::Error(QW_ERR_MODEL_LOAD, g_err);
        check_ids(target, prompt, n_prompt);
        QW_CUDA(cudaSetDevice(target->device));
        std::vector<int> p(prompt, prompt + n_prompt);
        qw::SpecRequest r;
        r.prompt = p.data();
        r.n_prompt = n_prompt;
        r.max_new = max_new;
        r.k = k;
        r.force_p = 0.f;
        r.seed = seed;
        r.forced = nullptr;
        r.n_forced = 0;
        r.eos_target = eos_list(target, eos, n_eos);
        r.eos_draft = eos_list(draft, eos, n_eos);
        r.temperature = temperature;
        r.top_p = top_p;
        std::vector<int> toks;
        qw_spec_stats s;
        std::memset(&s, 0, sizeof(s));
        qw::spec_generate_dev(target, draft, r, toks, &s);
        for (size_t i = 0; i < toks.size(); ++i) out[i] = (uint32_t)toks[i];
        *n_out = (int)toks.size();
        if (stats) *stats = s;
    });
}

// The multi-row qw_quantized_matmul keeps one fp16 activation buffer per
// (device, stream), grown on demand and kept until exit: calls on one stream
// are ordered, so they can share it, and no call pays an allocation.
static void* qmm_scratch(int dev, cudaStream_t st, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> bufs;
    std::lock_guard<std::mutex> lk(mu);
    auto& b = bufs[{dev, st}];
    if (b.second < bytes) {
        // growing the buffer synchronises and allocates, which a stream capture cannot hold
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QW_CUDA(cudaStreamIsCapturing(st, &cs));
        if (cs != cudaStreamCaptureStatusNone)
            throw qw::Error(QW_ERR_INVALID_ARG,
                            "qw_quantized_matmul: the stream is being captured and its activation buffer must grow "
                            "to " + std::to_string(bytes) + " bytes; make one call at the largest M before capturing");
        if (b.first) {
            QW_CUDA(cudaStreamSynchronize(st));  // the old buffer may still be read by earlier work
            cudaFree(b.first);
            b = {nullptr, 0};
        }
        void* p = nullptr;
        QW_CUDA(cudaMalloc(&p, bytes));
        b = {p, bytes};
    }
    return b.first;
}

// QW_PREFILL_GEMM=legacy keeps multi-row matmuls on the mma.sync kernel.
static bool legacy_prefill_gemm() {
    const char* e = std::getenv("QW_PREFILL_GEMM");
    return e && std::strcmp(e, "legacy") == 0;
}

int qw_quantized_matmul(const void* x, const void* w, const void* scales, const void* biases, void* y, int M,
                        int N, int K, int group_size, int bits, void* stream) {
    return guard([&] {
        need(x && w && scales && biases && y, "pointers");
        if (group_size != 64 || bits != 4)
            throw qw::Error(QW_ERR_UNSUPPORTED, "only group_size 64 / bits 4 are supported");
        need(M >= 1 && N >= 1 && K >= 64 && K % 64 == 0, "shape (K must be a positive multiple of 64)");
        int dev = 0, sms = 0;
        QW_CUDA(cudaGetDevice(&dev));
        QW_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        qw::QmmArgs a;
        std::memset(&a, 0, sizeof(a));
        a.x = (const bf16*)x;
        a.ldx = K;
        a.M = M;
        a.K = K;
        a.seg[0].w = (const uint32_t*)w;
        a.seg[0].s = (const bf16*)scales;
        a.seg[0].b = (const bf16*)biases;
        a.seg[0].y = y;
        a.seg[0].n = N;
        a.seg[0].ldy = N;
        a.nseg = 1;
        a.epi = qw::EPI_STORE;
        cudaStream_t st = (cudaStream_t)stream;
        if (M <= 8) {
            // programmatic launch: the GEMV's blocks start while the previous
            // kernel drains and prefetch their weights into L2; every read of
            // x, w, scales and biases into the SMs and every write of y follows
            // the wait on that kernel.  cudaErrorNotSupported: no GEMV form
            // fits this row length in shared memory, the tiled GEMM takes it.
            a.weights_after_wait = 1;
            const cudaError_t e = qw::launch_qgemv(a, st, true, sms);
            if (e != cudaErrorNotSupported) {
                QW_CUDA(e);
                return;
            }
            a.weights_after_wait = 0;
        }
        if (qw::qgemm_tc_supported(a) && !legacy_prefill_gemm()) {
            // fp16 copy of x for the tensor-core kernel, then (output tiles
            // fewer than the SMs) the fp32 partials of a K split
            const int ksplit = qw::qgemm_tc_ksplit(a, sms);
            const size_t bytes = ((qw::qgemm_tc_scratch_bytes(M, K) + 255) & ~(size_t)255) +
                                 qw::qgemm_tc_ksplit_bytes(a, ksplit);
            QW_CUDA(qw::launch_qgemm_tc(a, qmm_scratch(dev, st, bytes), bytes, st, ksplit));
        } else {
            QW_CUDA(qw::launch_qgemm(a, st, sms));
        }
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// qw_quantized_matmul_argmax_static: the lm_head GEMV + argmax with its
// per-CTA maxima in a static device array instead of a workspace allocation.
// ---------------------------------------------------------------------------
namespace {

// Slot (rb, m) = this row block's packed (logit, index) maximum of row m.
// Every slot the finalize kernel reads is written earlier by the same call, so
// nothing in it has to start at zero.
static __device__ __align__(256) unsigned long long g_static_amax[QW_STATIC_AMAX_SLOTS];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
unsigned long long* g_static_amax_ptr[kMaxDevices] = {};

// Address of g_static_amax on device `dev` (the current device), looked up on
// the first call for that device.
unsigned long long* static_amax(int dev) {
    if (dev < 0 || dev >= kMaxDevices) throw qw::Error(QW_ERR_INVALID_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_amax_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_amax);
        if (e != cudaSuccess || !p)
            throw qw::Error(QW_ERR_CUDA, std::string("cudaGetSymbolAddress(static argmax scratch): ") +
                                             cudaGetErrorString(e));
        g_static_amax_ptr[dev] = static_cast<unsigned long long*>(p);
    }
    return g_static_amax_ptr[dev];
}

}  // namespace

extern "C" int qw_quantized_matmul_argmax_static(const void* x, const void* w, const void* scales,
                                                 const void* biases, void* y_or_null, int* argmax_dev, int M,
                                                 int N, int K, int group_size, int bits, void* stream) {
    return guard([&] {
        need(x && w && scales && biases && argmax_dev, "pointers");
        if (group_size != 64 || bits != 4)
            throw qw::Error(QW_ERR_UNSUPPORTED, "only group_size 64 / bits 4 are supported");
        need(M >= 1 && M <= 8 && N >= 1 && K >= 64 && K % 64 == 0,
             "shape (1 <= M <= 8, N >= 1, K a positive multiple of 64)");
        const long long slots = (long long)M * ((N + 15) / 16);
        if (slots > QW_STATIC_AMAX_SLOTS)
            throw qw::Error(QW_ERR_INVALID_ARG, "qw_quantized_matmul_argmax_static: M * ceil(N/16) = " +
                                                    std::to_string(slots) + " exceeds the static scratch of " +
                                                    std::to_string(QW_STATIC_AMAX_SLOTS) + " slots");
        int dev = 0, sms = 0;
        QW_CUDA(cudaGetDevice(&dev));
        QW_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        unsigned long long* scratch = static_amax(dev);
        qw::QmmArgs a;
        std::memset(&a, 0, sizeof(a));
        a.x = (const bf16*)x;
        a.ldx = K;
        a.M = M;
        a.K = K;
        a.seg[0].w = (const uint32_t*)w;
        a.seg[0].s = (const bf16*)scales;
        a.seg[0].b = (const bf16*)biases;
        a.seg[0].y = y_or_null;
        a.seg[0].n = N;
        a.seg[0].ldy = N;
        a.nseg = 1;
        a.epi = qw::EPI_LOGITS;
        a.store_logits = y_or_null ? 1 : 0;
        a.amax_partial = scratch;
        if (!qw::qgemv_fits(a))
            throw qw::Error(QW_ERR_INVALID_ARG, "qw_quantized_matmul_argmax_static: K = " + std::to_string(K) +
                                                    " at M = " + std::to_string(M) +
                                                    " does not fit the GEMV's shared-memory staging (220 KB); "
                                                    "largest K: " + std::to_string(qw::qgemv_max_k(M)));
        cudaStream_t st = (cudaStream_t)stream;
        a.weights_after_wait = 1;  // programmatic launch with L2 hints only before the wait
        QW_CUDA(qw::launch_qgemv(a, st, true, sms));
        QW_CUDA(qw::launch_amax_finalize(scratch, qw::qgemv_row_blocks(a), M, argmax_dev, nullptr, st));
    });
}

