// comm.cpp -- head-parallel all-gather over NCCL (NVLink / NVSwitch).
//
// The reference has no collective: it renders on a single device
// (RenderEngine.swift:16-24).  Heads are independent, so a head-sharded job
// needs communication only where a caller wants every head's output on every
// rank; this file provides exactly that gather.
//
// NCCL is opened lazily with dlopen: a process that already loaded an NCCL
// (PyTorch bundles one) reuses it, and the library itself has no link-time
// NCCL dependency, so attention calls work where NCCL is absent.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ltxattn.h"
#include "ltxattn_internal.h"

namespace ltx {
int set_error_message(int status, const char* msg);
}

struct ltxattn_comm {
  ncclComm_t nccl;
  int nranks;
  int rank;
  int device;
};

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
  ncclResult_t (*CommCount)(const ncclComm_t, int*);
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*);
  bool ok;
};

const NcclApi& nccl() {
  static NcclApi api{};
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(h, "ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.CommCount = reinterpret_cast<decltype(api.CommCount)>(dlsym(h, "ncclCommCount"));
    api.CommUserRank = reinterpret_cast<decltype(api.CommUserRank)>(dlsym(h, "ncclCommUserRank"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllGather && api.AllReduce && api.GroupStart &&
             api.GroupEnd && api.GetErrorString && api.CommCount && api.CommUserRank;
  });
  return api;
}

int nccl_fail(const char* what, ncclResult_t r) {
  char buf[256];
  snprintf(buf, sizeof buf, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
  return ltx::set_error_message(LTXATTN_ERR_NCCL, buf);
}

int need_nccl() {
  if (!nccl().ok) return ltx::set_error_message(LTXATTN_ERR_NCCL, "libnccl.so.2 could not be loaded");
  return LTXATTN_OK;
}

}  // namespace

extern "C" {

int ltxattn_comm_unique_id(uint8_t id[128]) {
  if (!id) return ltx::set_error_message(LTXATTN_ERR_ARG, "id is NULL");
  if (int rc = need_nccl()) return rc;
  ncclUniqueId u;
  ncclResult_t r = nccl().GetUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  memcpy(id, u.internal, 128);
  return LTXATTN_OK;
}

int ltxattn_comm_init(ltxattn_comm** comm, int32_t nranks, int32_t rank, const uint8_t id[128], int32_t device) {
  if (!comm || !id) return ltx::set_error_message(LTXATTN_ERR_ARG, "comm or id is NULL");
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return ltx::set_error_message(LTXATTN_ERR_ARG, "rank out of range");
  if (int rc = need_nccl()) return rc;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // not left behind for a later launch check to find
    return ltx::set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  }
  ncclUniqueId u;
  memcpy(u.internal, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = nccl().CommInitRank(&c, nranks, u, rank);
  if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
  *comm = new ltxattn_comm{c, nranks, rank, device};
  return LTXATTN_OK;
}

int ltxattn_comm_destroy(ltxattn_comm* comm) {
  if (!comm) return LTXATTN_OK;
  int rc = LTXATTN_OK;
  if (nccl().ok && comm->nccl) {
    ncclResult_t r = nccl().CommDestroy(comm->nccl);
    if (r != ncclSuccess) rc = nccl_fail("ncclCommDestroy", r);
  }
  delete comm;
  return rc;
}

int ltxattn_comm_size(const ltxattn_comm* comm, int32_t* nranks, int32_t* rank) {
  if (!comm || !nranks || !rank) return ltx::set_error_message(LTXATTN_ERR_ARG, "comm, nranks or rank is NULL");
  if (int rc = need_nccl()) return rc;
  int n = 0, r = 0;
  ncclResult_t res = nccl().CommCount(comm->nccl, &n);
  if (res != ncclSuccess) return nccl_fail("ncclCommCount", res);
  res = nccl().CommUserRank(comm->nccl, &r);
  if (res != ncclSuccess) return nccl_fail("ncclCommUserRank", res);
  *nranks = n;
  *rank = r;
  return LTXATTN_OK;
}

int ltxattn_allgather_heads(const ltxattn_gather_args* a, ltxattn_comm* comm, void* stream) {
  if (!a || !comm) return ltx::set_error_message(LTXATTN_ERR_ARG, "args or comm is NULL");
  if (a->dtype != LTXATTN_F32 && a->dtype != LTXATTN_BF16)
    return ltx::set_error_message(LTXATTN_ERR_DTYPE, "dtype must be LTXATTN_F32 or LTXATTN_BF16");
  if (a->batch < 1 || a->heads_per_rank < 1 || a->tokens < 1 || a->head_dim < 1)
    return ltx::set_error_message(LTXATTN_ERR_SHAPE, "gather sizes must be >= 1");
  if (!a->send || !a->recv) return ltx::set_error_message(LTXATTN_ERR_ARG, "send or recv is NULL");
  if (int rc = need_nccl()) return rc;
  const size_t esize = a->dtype == LTXATTN_BF16 ? 2 : 4;
  const ncclDataType_t t = a->dtype == LTXATTN_BF16 ? ncclBfloat16 : ncclFloat32;
  const size_t count = (size_t)a->heads_per_rank * a->tokens * a->head_dim;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ncclResult_t r = nccl().GroupStart();
  if (r != ncclSuccess) return nccl_fail("ncclGroupStart", r);
  for (int b = 0; b < a->batch; ++b) {
    const char* s = static_cast<const char*>(a->send) + (size_t)b * count * esize;
    char* d = static_cast<char*>(a->recv) + (size_t)b * comm->nranks * count * esize;
    r = nccl().AllGather(s, d, count, t, comm->nccl, st);
    if (r != ncclSuccess) {
      nccl().GroupEnd();
      return nccl_fail("ncclAllGather", r);
    }
  }
  r = nccl().GroupEnd();
  if (r != ncclSuccess) return nccl_fail("ncclGroupEnd", r);
  return LTXATTN_OK;
}

size_t ltxattn_out_project_workspace(const ltxattn_out_project_args* a) {
  if (!a || a->m < 1 || a->n < 1) return 0;
  return ((size_t)a->m * a->n * sizeof(float) + 255) & ~size_t(255);
}

// Row-parallel to_out: this rank's heads' slice of the merged attention output
// times its column block of to_out.0.weight, as an fp32 partial in the
// workspace; the partials of all ranks summed in place by ncclAllReduce; then
// out = T(T(sum) + bias) on every rank.  All three steps are ordered on
// `stream`.  With one rank the result is bit-identical to ltxattn_linear.
int ltxattn_out_project_allreduce(const ltxattn_out_project_args* a, ltxattn_comm* comm, void* stream) {
  if (!a || !comm) return ltx::set_error_message(LTXATTN_ERR_ARG, "args or comm is NULL");
  if (a->dtype != LTXATTN_BF16)
    return ltx::set_error_message(LTXATTN_ERR_DTYPE, "ltxattn_out_project_allreduce: bf16 only");
  const size_t need = ltxattn_out_project_workspace(a);
  if (need == 0) return ltx::set_error_message(LTXATTN_ERR_SHAPE, "ltxattn_out_project_allreduce: m and n must be >= 1");
  if (!a->workspace || a->workspace_bytes < need || (reinterpret_cast<uintptr_t>(a->workspace) & 255u)) {
    char buf[200];
    snprintf(buf, sizeof buf, "ltxattn_out_project_allreduce: a 256-byte aligned workspace of %zu bytes is needed", need);
    return ltx::set_error_message(LTXATTN_ERR_WORKSPACE, buf);
  }
  if (!a->out || a->out_stride < a->n || (a->out_stride % 8) || (reinterpret_cast<uintptr_t>(a->out) & 15u) ||
      (a->bias && (reinterpret_cast<uintptr_t>(a->bias) & 15u)))
    return ltx::set_error_message(LTXATTN_ERR_ALIGN, "ltxattn_out_project_allreduce: out and bias need 16-byte aligned rows");
  if (int rc = need_nccl()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(a->workspace);
  ltxattn_linear_args l{};
  l.dtype = a->dtype;
  l.m = a->m;
  l.n = a->n;
  l.k = a->k;
  l.x = a->x;
  l.x_stride = a->x_stride;
  l.weight = a->weight;
  l.weight_stride = a->weight_stride;
  l.bias = nullptr;
  l.out = a->out;
  l.out_stride = a->out_stride;
  if (int rc = ltx::linear_partial_f32(&l, partial, st)) return rc;
  const ncclResult_t r =
      nccl().AllReduce(partial, partial, (size_t)a->m * a->n, ncclFloat32, ncclSum, comm->nccl, st);
  if (r != ncclSuccess) return nccl_fail("ncclAllReduce", r);
  return ltx::bias_round(partial, 1, 0, a->bias, a->out, a->out_stride, a->m, a->n, st);
}

int ltxattn_out_project_fused(const ltxattn_out_project_args* a, const ltxattn_reduce_peers* g, void* stream) {
  if (!a || !g) return ltx::set_error_message(LTXATTN_ERR_ARG, "args or peers is NULL");
  if (a->dtype != LTXATTN_BF16)
    return ltx::set_error_message(LTXATTN_ERR_DTYPE, "ltxattn_out_project_fused: bf16 only");
  if (a->m < 1 || a->n < 8 || a->n % 8)
    return ltx::set_error_message(LTXATTN_ERR_SHAPE, "ltxattn_out_project_fused: m >= 1 and n a multiple of 8");
  if (g->world < 2 || g->world > 8 || g->rank < 0 || g->rank >= g->world || g->epoch == 0)
    return ltx::set_error_message(LTXATTN_ERR_ARG, "ltxattn_out_project_fused: 2 to 8 ranks, a valid rank, epochs from 1");
  if (g->out[g->rank] != a->out)
    return ltx::set_error_message(LTXATTN_ERR_ARG, "ltxattn_out_project_fused: peers->out[rank] must be args->out");
  for (int d = 0; d < g->world; ++d)
    if (!g->recv[d] || !g->out[d] || !g->signals[d] || (reinterpret_cast<uintptr_t>(g->recv[d]) & 15u) ||
        (reinterpret_cast<uintptr_t>(g->out[d]) & 15u))
      return ltx::set_error_message(LTXATTN_ERR_ALIGN, "ltxattn_out_project_fused: 16-byte aligned peer buffers needed");
  if (a->out_stride < a->n || (a->out_stride % 8) || (a->bias && (reinterpret_cast<uintptr_t>(a->bias) & 15u)))
    return ltx::set_error_message(LTXATTN_ERR_ALIGN, "ltxattn_out_project_fused: out and bias need 16-byte aligned rows");
  int* err = ltx::device_error_word();
  if (!err) return ltx::set_error_message(LTXATTN_ERR_CUDA, "no device error word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int blocks = (a->m + 127) / 128;
  const int rows_per_owner = (blocks + g->world - 1) / g->world * 128;
  const int64_t slot = (int64_t)a->m * a->n;
  ltxattn_linear_args l{};
  l.dtype = a->dtype;
  l.m = a->m;
  l.n = a->n;
  l.k = a->k;
  l.x = a->x;
  l.x_stride = a->x_stride;
  l.weight = a->weight;
  l.weight_stride = a->weight_stride;
  l.out = a->out;
  l.out_stride = a->out_stride;
  // 1. every partial row into its owner's plane for this rank
  if (int rc = ltx::linear_partial_f32_to_owners(&l, g->recv, g->world, g->rank, rows_per_owner, slot, st)) return rc;
  ltx::GatherSync gs{};
  gs.n = g->world;
  gs.rank = g->rank;
  gs.epoch = g->epoch;
  gs.err = err;
  for (int d = 0; d < g->world; ++d) gs.sig[d] = g->signals[d];
  // 2. every rank's partials have landed at their owners
  gs.word = 0;
  cudaError_t e = ltx::launch_gather_done(gs, st);
  if (e != cudaSuccess) return ltx::set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  // 3. this rank's rows: planes added in rank order, bias and roundings, stored in every output
  const int r0 = g->rank * rows_per_owner;
  const int rows = std::max(0, std::min(a->m, r0 + rows_per_owner) - r0);
  void* peer_rows[7];
  int np = 0;
  for (int d = 0; d < g->world; ++d)
    if (d != g->rank) peer_rows[np++] = static_cast<__nv_bfloat16*>(g->out[d]) + (int64_t)r0 * a->out_stride;
  if (rows > 0)
    if (int rc = ltx::bias_round(g->recv[g->rank] + (int64_t)r0 * a->n, g->world, slot, a->bias,
                                 static_cast<__nv_bfloat16*>(a->out) + (int64_t)r0 * a->out_stride, a->out_stride, rows,
                                 a->n, st, np, peer_rows))
      return rc;
  // 4. every rank's rows have landed in every output
  gs.word = 8;
  e = ltx::launch_gather_done(gs, st);
  if (e != cudaSuccess) return ltx::set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  return LTXATTN_OK;
}

}  // extern "C"
