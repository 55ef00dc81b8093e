// comm.cu -- the multi-GPU exchanges of the sharded layer path behind the C ABI.
//
// The reference has no distributed runtime (plan.md:325 lists one as a
// stretch goal), so these entry points have no counterpart there: they are the
// collectives a native host (oxitorch's Rust crates) needs to run the sharded
// layers without Python -- the all-reduce of weight-gradient partials and of
// the cross-entropy loss, f64 sums of squares, the reduce-scatter of a table
// gradient and the variable all-to-all of the sparse embedding exchange.
//
// Transport: NCCL over NVLink / NVSwitch, loaded at run time (dlopen of
// libnccl.so.2), so the library has no link-time NCCL dependency and, inside a
// process that already loaded an NCCL (torch does), shares that one.  One
// communicator per process and GPU; every rank issues the same calls in the
// same order; every call is asynchronous on the caller's stream.
#include <cuda.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

struct oxc_comm {
  ncclComm_t nccl;
  int32_t world, rank, device;
};

namespace oxc {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t);
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  const char* (*error_string)(ncclResult_t);
  bool ok;
};

std::mutex g_nccl_mu;
NcclApi g_nccl{};
bool g_nccl_tried = false;
char g_nccl_error[256] = "";

template <typename T>
bool bind(void* h, const char* name, T* fn) {
  *fn = reinterpret_cast<T>(dlsym(h, name));
  return *fn != nullptr;
}

const NcclApi* nccl_api() {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (!g_nccl_tried) {
    g_nccl_tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      snprintf(g_nccl_error, sizeof g_nccl_error, "%s", dlerror());
    } else {
      NcclApi a{};
      a.ok = bind(h, "ncclGetUniqueId", &a.get_unique_id) &&
             bind(h, "ncclCommInitRank", &a.comm_init_rank) &&
             bind(h, "ncclCommDestroy", &a.comm_destroy) &&
             bind(h, "ncclAllReduce", &a.all_reduce) &&
             bind(h, "ncclReduceScatter", &a.reduce_scatter) && bind(h, "ncclSend", &a.send) &&
             bind(h, "ncclRecv", &a.recv) && bind(h, "ncclGroupStart", &a.group_start) &&
             bind(h, "ncclGroupEnd", &a.group_end) &&
             bind(h, "ncclGetErrorString", &a.error_string);
      if (!a.ok) snprintf(g_nccl_error, sizeof g_nccl_error, "libnccl.so.2 lacks a symbol");
      g_nccl = a;
    }
  }
  return g_nccl.ok ? &g_nccl : nullptr;
}

oxc_status nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
  return fail(OXC_ERR_OTHER, "%s: NCCL error %d (%s)", what, (int)r,
              api && api->error_string ? api->error_string(r) : "?");
}

oxc_status need_api(const NcclApi** api, const char* what) {
  *api = nccl_api();
  if (!*api) return fail(OXC_ERR_OTHER, "%s: NCCL is not available: %s", what, g_nccl_error);
  return OXC_OK;
}

oxc_status check_comm(const oxc_comm* comm, const char* what) {
  if (!comm || !comm->nccl)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null communicator", what);
  return OXC_OK;
}

}  // namespace
}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_comm_unique_id(uint8_t* id) {
  const char* fn = "oxc_comm_unique_id";
  if (!id) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null id", fn);
  static_assert(sizeof(ncclUniqueId) == OXC_COMM_ID_BYTES, "ncclUniqueId size");
  const NcclApi* api;
  oxc_status st = need_api(&api, fn);
  if (st) return st;
  ncclUniqueId u;
  ncclResult_t r = api->get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(api, r, fn);
  std::memcpy(id, &u, sizeof u);
  return OXC_OK;
}

oxc_status oxc_comm_init(oxc_comm** comm, const uint8_t* id, int32_t world, int32_t rank) {
  const char* fn = "oxc_comm_init";
  if (!comm || !id) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  *comm = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: rank %d of world %d", (int)rank,
                (int)world);
  const NcclApi* api;
  oxc_status st = need_api(&api, fn);
  if (st) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  ncclComm_t c = nullptr;
  ncclResult_t r = api->comm_init_rank(&c, world, u, rank);
  if (r != ncclSuccess) return nccl_fail(api, r, fn);
  *comm = new oxc_comm{c, world, rank, dev};
  return OXC_OK;
}

oxc_status oxc_comm_destroy(oxc_comm* comm) {
  if (!comm) return OXC_OK;
  const NcclApi* api;
  oxc_status st = need_api(&api, "oxc_comm_destroy");
  if (st) return st;
  ncclResult_t r = comm->nccl ? api->comm_destroy(comm->nccl) : ncclSuccess;
  delete comm;
  return r == ncclSuccess ? OXC_OK : nccl_fail(api, r, "oxc_comm_destroy");
}

static oxc_status allreduce(oxc_comm* comm, void* buf, int64_t n, ncclDataType_t t, void* stream,
                            const char* fn) {
  oxc_status st = check_comm(comm, fn);
  if (st) return st;
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative count", fn);
  if (n == 0) return OXC_OK;
  if (!buf) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null buffer", fn);
  const NcclApi* api;
  if ((st = need_api(&api, fn))) return st;
  ncclResult_t r = api->all_reduce(buf, buf, (size_t)n, t, ncclSum, comm->nccl,
                                   static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? OXC_OK : nccl_fail(api, r, fn);
}

oxc_status oxc_comm_allreduce_sum_f32(oxc_comm* comm, float* buf, int64_t n, void* stream) {
  return allreduce(comm, buf, n, ncclFloat32, stream, "oxc_comm_allreduce_sum_f32");
}

oxc_status oxc_comm_allreduce_sum_f64(oxc_comm* comm, double* buf, int64_t n, void* stream) {
  return allreduce(comm, buf, n, ncclFloat64, stream, "oxc_comm_allreduce_sum_f64");
}

oxc_status oxc_comm_reduce_scatter_f32(oxc_comm* comm, const float* in, float* out,
                                       int64_t count_per_rank, void* stream) {
  const char* fn = "oxc_comm_reduce_scatter_f32";
  oxc_status st = check_comm(comm, fn);
  if (st) return st;
  if (count_per_rank < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative count", fn);
  if (count_per_rank == 0) return OXC_OK;
  if (!in || !out) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null buffer", fn);
  const NcclApi* api;
  if ((st = need_api(&api, fn))) return st;
  ncclResult_t r = api->reduce_scatter(in, out, (size_t)count_per_rank, ncclFloat32, ncclSum,
                                       comm->nccl, static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? OXC_OK : nccl_fail(api, r, fn);
}

oxc_status oxc_comm_alltoallv(oxc_comm* comm, const void* send, const int64_t* send_counts,
                              void* recv, const int64_t* recv_counts, int64_t elem_bytes,
                              void* stream) {
  const char* fn = "oxc_comm_alltoallv";
  oxc_status st = check_comm(comm, fn);
  if (st) return st;
  if (!send_counts || !recv_counts || elem_bytes <= 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: counts", fn);
  const NcclApi* api;
  if ((st = need_api(&api, fn))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t soff = 0, roff = 0;
  for (int p = 0; p < comm->world; ++p) {
    if (send_counts[p] < 0 || recv_counts[p] < 0)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative count", fn);
    soff += send_counts[p];
    roff += recv_counts[p];
  }
  if ((soff && !send) || (roff && !recv))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null buffer", fn);
  // bytes as ncclUint8: any element type, counts in elements of elem_bytes
  ncclResult_t r = api->group_start();
  soff = roff = 0;
  for (int p = 0; p < comm->world && r == ncclSuccess; ++p) {
    const size_t sb = (size_t)send_counts[p] * (size_t)elem_bytes;
    const size_t rb = (size_t)recv_counts[p] * (size_t)elem_bytes;
    if (sb)
      r = api->send(static_cast<const char*>(send) + soff, sb, ncclUint8, p, comm->nccl, s);
    if (r == ncclSuccess && rb)
      r = api->recv(static_cast<char*>(recv) + roff, rb, ncclUint8, p, comm->nccl, s);
    soff += (int64_t)sb;
    roff += (int64_t)rb;
  }
  const ncclResult_t r2 = api->group_end();
  if (r != ncclSuccess) return nccl_fail(api, r, fn);
  return r2 == ncclSuccess ? OXC_OK : nccl_fail(api, r2, fn);
}

// ---- device memory shared between the processes of one node (CUDA IPC) ----------

static CUresult (*mem_range_fn())(CUdeviceptr*, size_t*, CUdeviceptr) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<Fn>(p);
  }();
  return fn;
}

oxc_status oxc_ipc_export(const void* dev_ptr, uint8_t* handle, int64_t* offset) {
  const char* fn = "oxc_ipc_export";
  if (!dev_ptr || !handle || !offset)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  static_assert(sizeof(cudaIpcMemHandle_t) == OXC_IPC_HANDLE_BYTES, "cudaIpcMemHandle_t size");
  auto range = mem_range_fn();
  if (!range) return fail(OXC_ERR_OTHER, "%s: cuMemGetAddressRange is not available", fn);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)(uintptr_t)dev_ptr) != CUDA_SUCCESS)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: not device memory", fn);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  std::memcpy(handle, &h, sizeof h);
  *offset = (int64_t)((uintptr_t)dev_ptr - (uintptr_t)base);
  return OXC_OK;
}

oxc_status oxc_ipc_import(const uint8_t* handle, int64_t offset, void** dev_ptr) {
  const char* fn = "oxc_ipc_import";
  if (!handle || !dev_ptr || offset < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: bad argument", fn);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  *dev_ptr = static_cast<char*>(base) + offset;
  return OXC_OK;
}

oxc_status oxc_ipc_close(void* dev_ptr, int64_t offset) {
  if (!dev_ptr) return OXC_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset);
  return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_ipc_close");
}

}  // extern "C"
