// NCCL plumbing of the row-sharded entry points (token rows shard across
// GPUs with replicated codebooks; the one exchange is an all-gather of codes
// and reconstructions over NVLink). NCCL is opened with dlopen on first use,
// so the library loads and runs single-GPU without it; a process that has
// already loaded libnccl (through PyTorch, say) shares that copy.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "internal.h"

namespace ncm {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    auto sym = [h](const char* n) { return dlsym(h, n); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.all_gather &&
             api.group_start && api.group_end && api.error_string;
  });
  return api;
}

int nccl_fail(const NcclApi& api, ncclResult_t r, const char* what) {
  return ncm_fail(NCM_ECUDA, "%s: NCCL error %d (%s)", what, static_cast<int>(r), api.error_string(r));
}

}  // namespace

int comm_all_gather(ncm_ctx* ctx, const AllGatherItem* items, int n, cudaStream_t stream) {
  const NcclApi& api = nccl();
  if (ctx->comm == nullptr || !api.ok) return ncm_fail(NCM_EINVAL, "no communicator bound (ncm_ctx_comm_init)");
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  ncclResult_t r = api.group_start();
  if (r != ncclSuccess) return nccl_fail(api, r, "all-gather");
  for (int i = 0; i < n; ++i) {
    // byte-wise transfer: any element type moves as count * bytes_per_elem bytes
    r = api.all_gather(items[i].send, items[i].recv, items[i].count * items[i].bytes_per_elem, ncclUint8, comm,
                       stream);
    if (r != ncclSuccess) break;
  }
  const ncclResult_t r2 = api.group_end();
  if (r != ncclSuccess) return nccl_fail(api, r, "all-gather");
  if (r2 != ncclSuccess) return nccl_fail(api, r2, "all-gather");
  return NCM_OK;
}

void comm_release(ncm_ctx* ctx) {
  if (ctx->comm == nullptr) return;
  const NcclApi& api = nccl();
  if (api.ok) api.comm_destroy(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
  ctx->comm_rank = 0;
  ctx->comm_size = 1;
}

}  // namespace ncm

using namespace ncm;

extern "C" {

int ncm_comm_unique_id(uint8_t* id_out) {
  if (id_out == nullptr) return ncm_fail(NCM_EINVAL, "comm_unique_id: null output");
  const NcclApi& api = nccl();
  if (!api.ok) return ncm_fail(NCM_ENOTSUP, "comm_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(api, r, "comm_unique_id");
  static_assert(sizeof(id) == NCCL_UNIQUE_ID_BYTES, "unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return NCM_OK;
}

int ncm_ctx_comm_init(ncm_ctx_t* ctx, const uint8_t* id, int32_t rank, int32_t nranks) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  if (id == nullptr) return ncm_fail(NCM_EINVAL, "comm_init: null id");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return ncm_fail(NCM_EINVAL, "comm_init: rank %d outside [0, %d)", rank, nranks);
  const NcclApi& api = nccl();
  if (!api.ok) return ncm_fail(NCM_ENOTSUP, "comm_init: libnccl.so.2 could not be loaded");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  comm_release(ctx);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  const ncclResult_t r = api.comm_init_rank(&comm, nranks, uid, rank);
  if (r != ncclSuccess) return nccl_fail(api, r, "comm_init");
  ctx->comm = comm;
  ctx->comm_rank = rank;
  ctx->comm_size = nranks;
  return NCM_OK;
}

}  // extern "C"
