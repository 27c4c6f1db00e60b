// Model construction: config parsing, weight arena, MLX safetensors loading,
// seeded random init, workspace and KV cache management.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <dirent.h>
#include <fstream>

#include "json.h"
#include "model.h"

namespace qw {

namespace {

int jint(const JValue* v, const char* name, bool required, int dflt) {
    if (!v || v->is_null()) {
        if (required) throw Error(QW_ERR_INVALID_CONFIG, std::string("config.json: missing field `") + name + "`");
        return dflt;
    }
    if (v->kind != JValue::NUM) throw Error(QW_ERR_INVALID_CONFIG, std::string("config.json: `") + name + "` is not a number");
    return (int)v->num;
}

uint64_t splitmix64_host(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
uint64_t tensor_key(uint64_t seed, uint64_t tid) { return splitmix64_host(seed ^ splitmix64_host(tid)); }
float normal_mult(double std) { return (float)(std / std::sqrt((4294967296.0 - 1.0) / 3.0)); }

// tensor ids shared with oracle/synth.py
constexpr int TID_EMBED = 0, TID_FINAL_NORM = 1, TID_LM_HEAD = 2;
enum { L_IN_NORM, L_Q, L_K, L_V, L_Q_NORM, L_K_NORM, L_O, L_POST_NORM, L_GATE, L_UP, L_DOWN };
int layer_tid(int l, int kind) { return 16 + 16 * l + kind; }

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// config.rs:149-201 (ModelConfig::from_path + validate + helpers).
Config parse_config(const std::string& text) {
    JValue j;
    try {
        j = json_parse(text);
    } catch (const std::exception& e) {
        throw Error(QW_ERR_INVALID_CONFIG, std::string("config.json: ") + e.what());
    }
    if (j.kind != JValue::OBJ) throw Error(QW_ERR_INVALID_CONFIG, "config.json: not an object");
    Config c;
    if (auto v = j.get("model_type")) c.model_type = v->kind == JValue::STR ? v->str : "";
    c.hidden = jint(j.get("hidden_size"), "hidden_size", true, 0);
    c.intermediate = jint(j.get("intermediate_size"), "intermediate_size", true, 0);
    c.layers = jint(j.get("num_hidden_layers"), "num_hidden_layers", true, 0);
    c.heads = jint(j.get("num_attention_heads"), "num_attention_heads", true, 0);
    c.vocab = jint(j.get("vocab_size"), "vocab_size", true, 0);
    if (c.hidden == 0 || c.heads == 0)
        throw Error(QW_ERR_INVALID_CONFIG, "hidden_size and num_attention_heads must be non-zero");
    c.kv_heads = jint(j.get("num_key_value_heads"), "num_key_value_heads", false, c.heads);
    const JValue* hd = j.get("head_dim");
    if ((!hd || hd->is_null()) && c.hidden % c.heads != 0)
        throw Error(QW_ERR_INVALID_CONFIG, "hidden_size (" + std::to_string(c.hidden) +
                                               ") not divisible by num_attention_heads (" + std::to_string(c.heads) +
                                               ") and no explicit head_dim");
    c.head_dim = jint(hd, "head_dim", false, c.hidden / c.heads);
    if (auto v = j.get("rms_norm_eps"); v && v->kind == JValue::NUM) c.eps = (float)v->num;
    if (auto v = j.get("rope_theta"); v && v->kind == JValue::NUM) c.rope_theta = (float)v->num;
    c.max_pos_emb = jint(j.get("max_position_embeddings"), "max_position_embeddings", false, 4096);
    if (auto v = j.get("tie_word_embeddings"); v && v->kind == JValue::BOOL) c.tied = v->b;
    if (auto v = j.get("bos_token_id"); v && v->kind == JValue::NUM) c.bos = (int)v->num;
    if (auto v = j.get("eos_token_id")) {
        if (v->kind == JValue::NUM) c.eos.push_back((int)v->num);
        if (v->kind == JValue::ARR)
            for (auto& e : v->arr)
                if (e.kind == JValue::NUM) c.eos.push_back((int)e.num);
    }
    // mlx-lm writes both `quantization` and `quantization_config`; prefer the first (config.rs:159-162)
    const JValue* q = j.get("quantization");
    if (!q || q->is_null()) q = j.get("quantization_config");
    if (q && q->kind == JValue::OBJ) {
        c.quantized = true;
        c.bits = jint(q->get("bits"), "quantization.bits", true, 0);
        c.group_size = jint(q->get("group_size"), "quantization.group_size", true, 0);
    }
    return c;
}

qw_model* model_create(const Config& cfg, int device, int tp_rank, int tp_size) {
    if (cfg.model_type != "qwen3")
        throw Error(QW_ERR_MODEL_LOAD, "unsupported model_type: " + cfg.model_type);
    if (!cfg.quantized) throw Error(QW_ERR_MODEL_LOAD, "only quantized models supported in v1");
    if (cfg.bits != 4 || cfg.group_size != 64)
        throw Error(QW_ERR_UNSUPPORTED, "only 4-bit group-64 affine quantization is supported (got bits=" +
                                            std::to_string(cfg.bits) + " group_size=" + std::to_string(cfg.group_size) + ")");
    if (cfg.head_dim != 128) throw Error(QW_ERR_UNSUPPORTED, "head_dim must be 128");
    if (cfg.hidden % 64 || cfg.intermediate % 64) throw Error(QW_ERR_UNSUPPORTED, "hidden/intermediate must be multiples of 64");
    if (cfg.kv_heads <= 0 || cfg.heads % cfg.kv_heads)
        throw Error(QW_ERR_INVALID_CONFIG, "num_attention_heads not a multiple of num_key_value_heads");
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) throw Error(QW_ERR_INVALID_ARG, "bad tp_rank/tp_size");
    if (cfg.heads % tp_size || cfg.kv_heads % tp_size || cfg.intermediate % (64 * tp_size) || cfg.vocab % tp_size)
        throw Error(QW_ERR_UNSUPPORTED, "heads / kv_heads / intermediate / vocab not divisible by tp_size");
    if (cfg.heads / cfg.kv_heads > 8) throw Error(QW_ERR_UNSUPPORTED, "GQA group larger than 8");
    int ndev = 0;
    QW_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) throw Error(QW_ERR_CUDA, "no such CUDA device: " + std::to_string(device));
    QW_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    QW_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) throw Error(QW_ERR_CUDA, std::string("this library is built for sm_100a; device is ") + prop.name);
    auto* m = new qw_model();
    m->cfg = cfg;
    m->device = device;
    m->tp_rank = tp_rank;
    m->tp_size = tp_size;
    m->hq_l = cfg.heads / tp_size;
    m->hkv_l = cfg.kv_heads / tp_size;
    m->inter_l = cfg.intermediate / tp_size;
    // tied heads stay replicated; an untied lm_head is split by vocabulary rows
    m->vocab_l = cfg.tied ? cfg.vocab : cfg.vocab / tp_size;
    m->num_sms = prop.multiProcessorCount;
    try {
        QW_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
        QW_CUDA(cudaMalloc(&m->d_err, sizeof(int)));
        QW_CUDA(cudaMemset(m->d_err, 0, sizeof(int)));
        // RoPE tables in float64 -> fp32 (angle = pos * theta^(-2i/D))
        m->rope_max_pos = std::min(std::max(4096, cfg.max_pos_emb), 65536);
        const int half = cfg.head_dim / 2;
        std::vector<float> cs((size_t)m->rope_max_pos * half), sn(cs.size());
        for (int i = 0; i < half; ++i) {
            const double inv = std::pow((double)cfg.rope_theta, (-2.0 * i) / (double)cfg.head_dim);
            for (int p = 0; p < m->rope_max_pos; ++p) {
                const double ang = (double)p * inv;
                cs[(size_t)p * half + i] = (float)std::cos(ang);
                sn[(size_t)p * half + i] = (float)std::sin(ang);
            }
        }
        QW_CUDA(cudaMalloc(&m->rope_cos, cs.size() * 4));
        QW_CUDA(cudaMalloc(&m->rope_sin, sn.size() * 4));
        QW_CUDA(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
        QW_CUDA(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
        model_alloc_weights(m);
    } catch (...) {
        delete m;
        throw;
    }
    return m;
}

// Lay out this rank's tensors in one device allocation and record them under
// their MLX names (qwen3.rs:205-273).
void model_alloc_weights(qw_model* m) {
    const Config& c = m->cfg;
    const int H = c.hidden, D = c.head_dim;
    struct Item {
        std::string name;
        size_t bytes;
        void** slot;
    };
    std::vector<Item> items;
    auto add = [&](const std::string& n, size_t bytes, void** slot) { items.push_back({n, bytes, slot}); };
    auto addq = [&](const std::string& p, QLin& q, int n, int k) {
        q.n = n;
        q.k = k;
        add(p + ".weight", (size_t)n * k / 2, (void**)&q.w);
        add(p + ".scales", (size_t)n * (k / 64) * 2, (void**)&q.s);
        add(p + ".biases", (size_t)n * (k / 64) * 2, (void**)&q.b);
    };
    addq("model.embed_tokens", m->embed, c.vocab, H);
    m->layers.resize(c.layers);
    for (int i = 0; i < c.layers; ++i) {
        Layer& L = m->layers[i];
        const std::string p = "model.layers." + std::to_string(i);
        add(p + ".input_layernorm.weight", (size_t)H * 2, (void**)&L.in_norm);
        add(p + ".post_attention_layernorm.weight", (size_t)H * 2, (void**)&L.post_norm);
        add(p + ".self_attn.q_norm.weight", (size_t)D * 2, (void**)&L.q_norm);
        add(p + ".self_attn.k_norm.weight", (size_t)D * 2, (void**)&L.k_norm);
        addq(p + ".self_attn.q_proj", L.q, m->hq_l * D, H);
        addq(p + ".self_attn.k_proj", L.k, m->hkv_l * D, H);
        addq(p + ".self_attn.v_proj", L.v, m->hkv_l * D, H);
        addq(p + ".self_attn.o_proj", L.o, H, m->hq_l * D);
        addq(p + ".mlp.gate_proj", L.gate, m->inter_l, H);
        addq(p + ".mlp.up_proj", L.up, m->inter_l, H);
        addq(p + ".mlp.down_proj", L.down, H, m->inter_l);
    }
    add("model.norm.weight", (size_t)H * 2, (void**)&m->final_norm);
    if (!c.tied) addq("lm_head", m->lm_head, m->vocab_l, H);
    size_t total = 0;
    for (auto& it : items) total += align256(it.bytes);
    QW_CUDA(cudaMalloc(&m->arena, total));
    m->arena_bytes = total;
    size_t off = 0;
    for (auto& it : items) {
        *it.slot = (char*)m->arena + off;
        m->tensors[it.name] = TensorRef{*it.slot, it.bytes};
        off += align256(it.bytes);
    }
    if (c.tied) m->lm_head = m->embed;
}

// ---- MLX safetensors loading ----------------------------------------------
namespace {

struct StEntry {
    std::string file;
    std::string dtype;
    std::vector<int64_t> shape;
    size_t begin = 0, end = 0;  // absolute file offsets
};

std::map<std::string, StEntry> scan_safetensors(const std::string& dir) {
    DIR* d = opendir(dir.c_str());
    if (!d) throw Error(QW_ERR_MODEL_LOAD, "cannot open model directory: " + dir);
    std::vector<std::string> files;
    while (dirent* e = readdir(d)) {
        std::string n = e->d_name;
        if (n.size() > 12 && n.substr(n.size() - 12) == ".safetensors") files.push_back(dir + "/" + n);
    }
    closedir(d);
    std::sort(files.begin(), files.end());
    if (files.empty()) throw Error(QW_ERR_MODEL_LOAD, "no .safetensors in " + dir);
    std::map<std::string, StEntry> out;
    for (auto& f : files) {
        std::ifstream in(f, std::ios::binary);
        uint64_t n = 0;
        in.read((char*)&n, 8);
        if (!in || n > (1ull << 30)) throw Error(QW_ERR_MODEL_LOAD, "load " + f + ": bad header");
        std::string hdr(n, '\0');
        in.read(&hdr[0], (std::streamsize)n);
        if (!in) throw Error(QW_ERR_MODEL_LOAD, "load " + f + ": truncated header");
        in.seekg(0, std::ios::end);
        const size_t fsize = (size_t)in.tellg();
        JValue j;
        try {
            j = json_parse(hdr);
        } catch (const std::exception& e) {
            throw Error(QW_ERR_MODEL_LOAD, "load " + f + ": " + e.what());
        }
        for (auto& kv : j.obj) {
            if (kv.first == "__metadata__") continue;
            StEntry s;
            s.file = f;
            if (auto dt = kv.second.get("dtype")) s.dtype = dt->str;
            if (auto sh = kv.second.get("shape"))
                for (auto& x : sh->arr) s.shape.push_back((int64_t)x.num);
            auto off = kv.second.get("data_offsets");
            if (!off || off->arr.size() != 2) throw Error(QW_ERR_MODEL_LOAD, "load " + f + ": bad data_offsets");
            s.begin = 8 + n + (size_t)off->arr[0].num;
            s.end = 8 + n + (size_t)off->arr[1].num;
            if (s.end < s.begin || s.end > fsize) throw Error(QW_ERR_MODEL_LOAD, "load " + f + ": data_offsets out of file");
            out[kv.first] = s;
        }
    }
    return out;
}

void read_bytes(const StEntry& e, std::vector<char>& buf) {
    buf.resize(e.end - e.begin);
    std::ifstream in(e.file, std::ios::binary);
    in.seekg((std::streamoff)e.begin);
    in.read(buf.data(), (std::streamsize)buf.size());
    if (!in) throw Error(QW_ERR_MODEL_LOAD, "load " + e.file + ": short read");
}

}  // namespace

// Qwen3::load (qwen3.rs:194-295): every expected tensor must be present
// ("missing tensor: ...") and nothing may be left over ("N unmapped tensors
// remain ...").  With tp_size > 1 only this rank's shard is uploaded.
void model_load_dir(qw_model* m, const std::string& dir) {
    auto st = scan_safetensors(dir);
    const Config& c = m->cfg;
    const int D = c.head_dim;
    std::vector<char> buf;
    auto shard_of = [&](const std::string& name, int64_t& r0, int64_t& rn, int64_t& c0, int64_t& cn, int64_t rows,
                        int64_t cols) {
        r0 = 0; rn = rows; c0 = 0; cn = cols;
        if (m->tp_size == 1) return;
        auto has = [&](const char* s) { return name.find(s) != std::string::npos; };
        if (has("q_proj.")) { rn = (int64_t)m->hq_l * D; r0 = rn * m->tp_rank; }
        else if (has("k_proj.") || has("v_proj.")) { rn = (int64_t)m->hkv_l * D; r0 = rn * m->tp_rank; }
        else if (has("gate_proj.") || has("up_proj.")) { rn = m->inter_l; r0 = rn * m->tp_rank; }
        else if (has("lm_head.")) { rn = m->vocab_l; r0 = rn * m->tp_rank; }
        else if (has("o_proj.") || has("down_proj.")) { cn = cols / m->tp_size; c0 = cn * m->tp_rank; }
    };
    std::map<std::string, bool> used;
    for (auto& kv : m->tensors) {
        const std::string& name = kv.first;
        auto it = st.find(name);
        if (it == st.end()) throw Error(QW_ERR_MODEL_LOAD, "missing tensor: " + name);
        used[name] = true;
        const StEntry& e = it->second;
        const bool is_w = e.dtype == "U32";
        const size_t esz = is_w ? 4 : 2;
        if (!is_w && e.dtype != "BF16")
            throw Error(QW_ERR_MODEL_LOAD, name + ": expected BF16 or U32 (got " + e.dtype + ")");
        const int64_t rows = e.shape.size() == 2 ? e.shape[0] : 1;
        const int64_t cols = e.shape.size() == 2 ? e.shape[1] : (e.shape.empty() ? 0 : e.shape[0]);
        if ((size_t)(rows * cols) * esz != e.end - e.begin)
            throw Error(QW_ERR_MODEL_LOAD, name + ": size does not match shape");
        int64_t r0, rn, c0, cn;
        shard_of(name, r0, rn, c0, cn, rows, cols);
        const size_t want = (size_t)(rn * cn) * esz;
        if (want != kv.second.bytes || r0 + rn > rows || c0 + cn > cols)
            throw Error(QW_ERR_MODEL_LOAD, name + ": shape mismatch with config (file has " +
                                               std::to_string(e.end - e.begin) + " bytes, this shard needs " +
                                               std::to_string(kv.second.bytes) + ")");
        read_bytes(e, buf);
        QW_CUDA(cudaMemcpy2D(kv.second.ptr, (size_t)cn * esz, buf.data() + ((size_t)r0 * cols + c0) * esz,
                             (size_t)cols * esz, (size_t)cn * esz, (size_t)rn, cudaMemcpyHostToDevice));
    }
    std::vector<std::string> left;
    for (auto& kv : st)
        if (!used.count(kv.first)) left.push_back(kv.first);
    if (!left.empty()) {
        std::string s = std::to_string(left.size()) + " unmapped tensors remain (first 5: [";
        for (size_t i = 0; i < left.size() && i < 5; ++i) s += (i ? ", \"" : "\"") + left[i] + "\"";
        throw Error(QW_ERR_MODEL_LOAD, s + "])");
    }
}

// ---- seeded random init (same bits as oracle/synth.py) ------------------
void model_init_random(qw_model* m, uint64_t seed, int norm_mode) {
    const Config& c = m->cfg;
    const int D = c.head_dim, H = c.hidden;
    const float mw = normal_mult(0.02), mn = normal_mult(0.1);
    cudaStream_t st = m->stream;
    auto q = [&](QLin& ql, int tid, int row0, int k0, int kfull) {
        QW_CUDA(launch_init_qweight(ql.w, ql.s, ql.b, ql.n, ql.k, row0, k0, kfull, tensor_key(seed, tid), mw, st));
    };
    auto nrm = [&](bf16* w, int n, int tid) {
        QW_CUDA(launch_init_norm(w, n, tensor_key(seed, tid), mn, norm_mode == 0, st));
    };
    const int r = m->tp_rank;
    q(m->embed, TID_EMBED, 0, 0, H);
    for (int i = 0; i < c.layers; ++i) {
        Layer& L = m->layers[i];
        nrm(L.in_norm, H, layer_tid(i, L_IN_NORM));
        nrm(L.post_norm, H, layer_tid(i, L_POST_NORM));
        nrm(L.q_norm, D, layer_tid(i, L_Q_NORM));
        nrm(L.k_norm, D, layer_tid(i, L_K_NORM));
        q(L.q, layer_tid(i, L_Q), r * m->hq_l * D, 0, H);
        q(L.k, layer_tid(i, L_K), r * m->hkv_l * D, 0, H);
        q(L.v, layer_tid(i, L_V), r * m->hkv_l * D, 0, H);
        q(L.o, layer_tid(i, L_O), 0, r * m->hq_l * D, c.heads * D);
        q(L.gate, layer_tid(i, L_GATE), r * m->inter_l, 0, H);
        q(L.up, layer_tid(i, L_UP), r * m->inter_l, 0, H);
        q(L.down, layer_tid(i, L_DOWN), 0, r * m->inter_l, c.intermediate);
    }
    nrm(m->final_norm, H, TID_FINAL_NORM);
    if (!c.tied) q(m->lm_head, TID_LM_HEAD, r * m->vocab_l, 0, H);
    QW_CUDA(cudaStreamSynchronize(st));
}

// ---- workspace -----------------------------------------------------------
void ensure_workspace(qw_model* m, int rows, int logits_rows) {
    Workspace& w = m->ws;
    rows = std::max(rows, 8);
    logits_rows = std::max(logits_rows, 8);
    if (rows <= w.cap_rows && logits_rows <= w.cap_logits && w.amax_partial) return;
    QW_CUDA(cudaStreamSynchronize(m->stream));
    for (void* p : w.allocs) cudaFree(p);
    w.allocs.clear();
    rows = std::max(rows, w.cap_rows);
    logits_rows = std::max(logits_rows, w.cap_logits);
    const Config& c = m->cfg;
    const size_t H = c.hidden, QD = (size_t)m->hq_l * c.head_dim, KD = (size_t)m->hkv_l * c.head_dim;
    auto alloc = [&](size_t bytes) {
        void* p = nullptr;
        QW_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
        w.allocs.push_back(p);
        return p;
    };
    w.x = (bf16*)alloc(rows * H * 2);
    w.h = (bf16*)alloc(rows * H * 2);
    w.q = (bf16*)alloc(rows * QD * 2);
    w.k = (bf16*)alloc(rows * KD * 2);
    w.v = (bf16*)alloc(rows * KD * 2);
    w.qr = (bf16*)alloc(rows * QD * 2);
    w.attn = (bf16*)alloc(rows * QD * 2);
    w.mlp = (bf16*)alloc(rows * (size_t)m->inter_l * 2);
    w.logits = (bf16*)alloc((size_t)logits_rows * m->vocab_l * 2);
    w.f32 = (float*)alloc(rows * H * 4);
    {
        const int kmax = std::max<int>((int)std::max(H, QD), m->inter_l);
        w.xh_bytes = qgemm_tc_scratch_bytes(rows, kmax);
        w.xh = alloc(w.xh_bytes);
    }
    w.ids = (int*)alloc(rows * 4);
    w.argmax = (int*)alloc(rows * 4);
    const size_t nrb_max = (size_t)m->vocab_l / 16 + 64;
    w.amax_partial = (unsigned long long*)alloc(nrb_max * 8 * 8);
    w.amax_keys = (unsigned long long*)alloc((size_t)logits_rows * 8);
    const int nsplit_max = std::max(1, 2 * m->num_sms);
    w.attn_part = (float*)alloc((size_t)m->hkv_l * nsplit_max * 64 * 130 * 4);
    // [sequence][query head]: one merge counter per (kv head, first query head of an item)
    w.attn_counters = (unsigned*)alloc((size_t)8 * std::max(m->hq_l, 8) * 4);
    w.next_tok = (int*)alloc(64);
    w.out_cap = std::max(w.out_cap, 65536);
    w.out = (int*)alloc((size_t)w.out_cap * 4);
    w.ctl = (StepCtl*)alloc(sizeof(StepCtl));
    w.bctl = (BatchCtl*)alloc(sizeof(BatchCtl));
    w.probs = (float*)alloc((size_t)m->vocab_l * 4);
    w.scfg = (SampleCfg*)alloc(sizeof(SampleCfg));
    w.sctrl = alloc(QW_SAMPLE_CTRL_BYTES);
    QW_CUDA(cudaMemset(w.sctrl, 0, QW_SAMPLE_CTRL_BYTES));
    QW_CUDA(cudaMemset(w.attn_counters, 0, (size_t)8 * std::max(m->hq_l, 8) * 4));
    QW_CUDA(cudaMemset(w.next_tok, 0, 64));
    w.cap_rows = rows;
    w.cap_logits = logits_rows;
    w.generation += 1;
}

qw_cache* cache_create(qw_model* m, int max_pos) {
    if (max_pos < 1 || max_pos > m->rope_max_pos)
        throw Error(QW_ERR_INVALID_ARG, "max_pos must be in [1, " + std::to_string(m->rope_max_pos) + "]");
    QW_CUDA(cudaSetDevice(m->device));
    auto* c = new qw_cache();
    c->m = m;
    c->max_pos = max_pos;
    const size_t n = (size_t)m->cfg.layers * m->hkv_l * max_pos * m->cfg.head_dim;
    try {
        QW_CUDA(cudaMalloc(&c->k, n * 2));
        QW_CUDA(cudaMalloc(&c->v, n * 2));
        QW_CUDA(cudaMalloc(&c->d_seq_len, sizeof(int)));
        QW_CUDA(cudaMemset(c->k, 0, n * 2));
        QW_CUDA(cudaMemset(c->v, 0, n * 2));
        QW_CUDA(cudaMemset(c->d_seq_len, 0, sizeof(int)));
    } catch (...) {
        delete c;
        throw;
    }
    m->caches.push_back(c);
    return c;
}

// generate() uses a model-owned cache of KV_PREALLOC = 4096 positions
// (qwen3.rs:125), grown when a request needs more; it is reset, not freed,
// between requests (the pre-allocation replaces MLX's allocator cache).
qw_cache* cache_for_generate(qw_model* m, int need_pos) {
    if (m->gen_cache && m->gen_cache->max_pos >= need_pos) return m->gen_cache;
    if (m->gen_cache) {
        qw_cache* old = m->gen_cache;
        m->gen_cache = nullptr;
        for (auto it = m->caches.begin(); it != m->caches.end(); ++it)
            if (*it == old) {
                m->caches.erase(it);
                break;
            }
        QW_CUDA(cudaStreamSynchronize(m->stream));
        delete old;
    }
    m->gen_cache = cache_create(m, std::min(std::max(4096, need_pos), m->rope_max_pos));
    return m->gen_cache;
}

void set_cache_len(qw_cache* c, int len) {
    QW_CUDA(cudaMemcpyAsync(c->d_seq_len, &len, sizeof(int), cudaMemcpyHostToDevice, c->m->stream));
    QW_CUDA(cudaStreamSynchronize(c->m->stream));
    c->seq_len = len;
}

void check_device_err(qw_model* m) {
    int e = 0;
    QW_CUDA(cudaMemcpy(&e, m->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        QW_CUDA(cudaMemset(m->d_err, 0, sizeof(int)));
        std::string what;
        if (e & QW_DERR_KV_RANGE) what += " kv-position-out-of-range";
        if (e & QW_DERR_TOKEN_RANGE) what += " token-id-out-of-range";
        if (e & QW_DERR_SHAPE) what += " unsupported-shape";
        throw Error(QW_ERR_DEVICE_FLAG, "device error flag set:" + what);
    }
}

}  // namespace qw

qw_model::~qw_model() {
    if (device >= 0) cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    // graphs that captured NCCL calls (the caches' step graphs, the spec graphs)
    // go before the communicator they use
    qw::spec_state_free(spec_state);
    spec_state = nullptr;
    for (qw_cache* c : caches) delete c;
    caches.clear();
    qw::tp_destroy(this);
    qw::mk_free(this);
    for (void* p : ws.allocs) cudaFree(p);
    if (arena) cudaFree(arena);
    if (rope_cos) cudaFree(rope_cos);
    if (rope_sin) cudaFree(rope_sin);
    if (d_err) cudaFree(d_err);
    if (stream) cudaStreamDestroy(stream);
}

qw_cache::~qw_cache() {
    if (step_graph) cudaGraphExecDestroy(step_graph);
    if (sample_graph) cudaGraphExecDestroy(sample_graph);
    if (k) cudaFree(k);
    if (v) cudaFree(v);
    if (d_seq_len) cudaFree(d_seq_len);
}

bf16* qw_cache::kl(int layer) const {
    return k + (size_t)layer * m->hkv_l * max_pos * m->cfg.head_dim;
}
bf16* qw_cache::vl(int layer) const {
    return v + (size_t)layer * m->hkv_l * max_pos * m->cfg.head_dim;
}
