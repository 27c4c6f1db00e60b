// Tensor-parallel communication for the large configs (Qwen3-32B over 2/4/8
// GPUs): one all-reduce (sum, fp32 partials) after o_proj and after down_proj,
// and a max-all-reduce of packed (logit, index) keys for the vocab-parallel
// lm_head.  The reference has no distributed path (ROADMAP.md:74-79); this is
// the split the benchmark's config 5 asks for.
//
// NCCL is resolved at attach time with dlopen, so the library itself loads on
// machines without NCCL; a model with tp_size > 1 fails loudly until
// qw_model_tp_attach has succeeded.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>

#include "model.h"

namespace qw {

struct TpComm {
    void* lib = nullptr;
    ncclComm_t comm = nullptr;
    ncclResult_t (*init)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allreduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    const char* (*errstr)(ncclResult_t) = nullptr;
};

static void* nccl_lib() {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char* n : names)
        if (void* h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) return h;
    return nullptr;
}

void tp_unique_id(void* out, size_t bytes) {
    if (bytes < sizeof(ncclUniqueId)) throw Error(QW_ERR_INVALID_ARG, "unique id buffer smaller than 128 bytes");
    void* lib = nccl_lib();
    if (!lib) throw Error(QW_ERR_CUDA, "cannot dlopen libnccl.so.2");
    auto get = (ncclResult_t(*)(ncclUniqueId*))dlsym(lib, "ncclGetUniqueId");
    if (!get) throw Error(QW_ERR_CUDA, "libnccl is missing ncclGetUniqueId");
    ncclUniqueId id;
    const ncclResult_t r = get(&id);
    if (r != ncclSuccess) throw Error(QW_ERR_CUDA, "ncclGetUniqueId failed");
    std::memcpy(out, &id, sizeof(id));
}

void tp_attach(qw_model* m, const void* unique_id, int rank, int size) {
    if (size != m->tp_size || rank != m->tp_rank)
        throw Error(QW_ERR_INVALID_ARG, "tp rank/size differ from the ones the model was loaded with");
    if (m->tp) throw Error(QW_ERR_INVALID_ARG, "communicator already attached");
    auto* t = new TpComm();
    t->lib = nccl_lib();
    if (!t->lib) {
        delete t;
        throw Error(QW_ERR_CUDA, "cannot dlopen libnccl.so.2");
    }
    t->init = (decltype(t->init))dlsym(t->lib, "ncclCommInitRank");
    t->allreduce = (decltype(t->allreduce))dlsym(t->lib, "ncclAllReduce");
    t->destroy = (decltype(t->destroy))dlsym(t->lib, "ncclCommDestroy");
    t->errstr = (decltype(t->errstr))dlsym(t->lib, "ncclGetErrorString");
    if (!t->init || !t->allreduce || !t->destroy || !t->errstr) {
        delete t;
        throw Error(QW_ERR_CUDA, "libnccl is missing required symbols");
    }
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    QW_CUDA(cudaSetDevice(m->device));
    ncclResult_t r = t->init(&t->comm, size, id, rank);
    if (r != ncclSuccess) {
        std::string msg = std::string("ncclCommInitRank: ") + t->errstr(r);
        delete t;
        throw Error(QW_ERR_CUDA, msg);
    }
    m->tp = t;
}

static void check_nccl(TpComm* t, ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw Error(QW_ERR_CUDA, std::string(what) + ": " + t->errstr(r));
}

void tp_allreduce_sum_f32(qw_model* m, float* buf, size_t count, cudaStream_t st) {
    if (!m->tp) throw Error(QW_ERR_INFERENCE, "tensor-parallel model has no communicator (call qw_model_tp_attach)");
    check_nccl(m->tp, m->tp->allreduce(buf, buf, count, ncclFloat32, ncclSum, m->tp->comm, st), "ncclAllReduce(sum)");
}

void tp_allreduce_max_u64(qw_model* m, unsigned long long* buf, size_t count, cudaStream_t st) {
    if (!m->tp) throw Error(QW_ERR_INFERENCE, "tensor-parallel model has no communicator (call qw_model_tp_attach)");
    check_nccl(m->tp, m->tp->allreduce(buf, buf, count, ncclUint64, ncclMax, m->tp->comm, st), "ncclAllReduce(max)");
}

void tp_destroy(qw_model* m) {
    if (!m->tp) return;
    if (m->tp->comm) m->tp->destroy(m->tp->comm);
    delete m->tp;
    m->tp = nullptr;
}

}  // namespace qw
