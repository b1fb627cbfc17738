// tp.cc -- tensor parallelism for the 7B-class models: the Megatron shard plan
// and the NCCL collectives the decode step uses.
//
// Sharding (per rank r of a world of W):
//   * column-parallel wq/wk/wv (+ bias) by head: query heads
//     [r*Hq/W, (r+1)*Hq/W) and key/value heads [r*Hkv/W, ...), so each rank's
//     grouped-query attention and KV cache stay local;
//   * column-parallel w_gate/w_up by FFN row [r*F/W, (r+1)*F/W);
//   * row-parallel wo and w_down split along K at 32-value block boundaries
//     (the matching query-head columns / FFN columns); each rank's product is
//     a partial sum, completed by one NCCL all-reduce (fp32, sum) per GEMV;
//   * vocab-parallel lm_head: rows [r*ceil(V/W), ...); greedy decoding takes
//     an all-reduce max over packed (value, index) keys, logits requested by
//     the host are all-gathered.
//   * embedding, norms and biases of row-parallel outputs replicated.
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"): a process that already
// holds torch's NCCL gets that copy, a plain C process the system one, and
// the library itself links against neither.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "dqmk.h"
#include "internal.h"
#include "tp.h"

namespace dqmk {
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("libnccl.so.2 not loadable: ") + (e ? e : "unknown");
      return;
    }
    auto sym = [&](const char* name) -> void* {
      void* p = dlsym(h, name);
      if (!p && api.why.empty()) api.why = std::string("NCCL symbol missing: ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.why.empty();
  });
  return api;
}

int nccl_fail(const char* api, ncclResult_t r) {
  const NcclApi& n = nccl();
  return fail(DQMK_ERR_CUDA, std::string(api) + ": NCCL error: " +
                                 (n.error_string ? n.error_string(r) : std::to_string((int)r)));
}

}  // namespace

int tp_plan(const dqmk_model_config& c, int rank, int world, dqmk_tp_plan* out) {
  const char* api = "dqmk_tp_plan_get";
  if (world < 1 || rank < 0 || rank >= world)
    return fail(DQMK_ERR_INVALID, std::string(api) + ": invalid rank or world size");
  const int qd = c.n_heads * c.head_dim;
  if (c.n_heads % world || c.n_kv_heads % world || c.hidden_dim % (32 * world) ||
      qd % (32 * world))
    return fail(DQMK_ERR_UNSUPPORTED,
                std::string(api) + ": heads, key/value heads, FFN width and query width must "
                                   "split evenly (FFN and query width at 32-value blocks)");
  dqmk_tp_plan p{};
  p.rank = rank;
  p.world = world;
  p.n_q_heads = c.n_heads / world;
  p.q_head0 = rank * p.n_q_heads;
  p.n_kv_heads = c.n_kv_heads / world;
  p.kv_head0 = rank * p.n_kv_heads;
  p.hidden = c.hidden_dim / world;
  p.hidden0 = rank * p.hidden;
  const int vl = (c.vocab_size + world - 1) / world;
  p.vocab0 = rank * vl;
  p.vocab = std::max(0, std::min(vl, c.vocab_size - p.vocab0));
  p.vocab_stride = vl;
  if (p.vocab <= 0)
    return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": vocabulary smaller than the world");
  *out = p;
  return DQMK_OK;
}

int tp_comm_create(int rank, int world, const unsigned char id[128], void** comm) {
  const char* api = "dqmk_model_set_tp";
  const NcclApi& n = nccl();
  if (!n.ok) return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": " + n.why);
  ncclUniqueId uid;
  static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(&uid, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = n.comm_init_rank(&c, world, uid, rank);
  if (r != ncclSuccess) return nccl_fail(api, r);
  *comm = c;
  return DQMK_OK;
}

void tp_comm_destroy(void* comm) {
  if (comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(comm));
}

int tp_allreduce_sum(void* comm, float* buf, size_t count, cudaStream_t s, const char* api) {
  ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum,
                                     static_cast<ncclComm_t>(comm), s);
  return r == ncclSuccess ? DQMK_OK : nccl_fail(api, r);
}

int tp_allreduce_max_u64(void* comm, unsigned long long* buf, size_t count, cudaStream_t s,
                         const char* api) {
  ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclUint64, ncclMax,
                                     static_cast<ncclComm_t>(comm), s);
  return r == ncclSuccess ? DQMK_OK : nccl_fail(api, r);
}

int tp_allgather(void* comm, const float* send, float* recv, size_t count, cudaStream_t s,
                 const char* api) {
  ncclResult_t r = nccl().all_gather(send, recv, count, ncclFloat32,
                                     static_cast<ncclComm_t>(comm), s);
  return r == ncclSuccess ? DQMK_OK : nccl_fail(api, r);
}

}  // namespace dqmk

using namespace dqmk;

extern "C" int dqmk_tp_plan_get(const dqmk_model_config* config, int rank, int world,
                                dqmk_tp_plan* out) {
  if (!config || !out) return fail(DQMK_ERR_INVALID, "dqmk_tp_plan_get: null argument");
  return tp_plan(*config, rank, world, out);
}

extern "C" int dqmk_nccl_unique_id(unsigned char* id_out) {
  const char* api = "dqmk_nccl_unique_id";
  if (!id_out) return fail(DQMK_ERR_INVALID, std::string(api) + ": null argument");
  const NcclApi& n = nccl();
  if (!n.ok) return fail(DQMK_ERR_UNSUPPORTED, std::string(api) + ": " + n.why);
  ncclUniqueId uid;
  ncclResult_t r = n.get_unique_id(&uid);
  if (r != ncclSuccess) return nccl_fail(api, r);
  std::memcpy(id_out, &uid, 128);
  return DQMK_OK;
}
