// fw_ep.cu -- the collectives of expert parallelism, over NCCL.
//
// With expert parallelism, rank r of N holds the experts e with e % N == r
// of every layer and brings its own T tokens to each forward.  A layer then
// moves data twice (the block's only exchange steps):
//   dispatch: every rank's token rows, top-k ids and route weights are
//             gathered on every rank (three all-gathers in one NCCL group);
//   combine:  the weighted expert rows computed for rank d's tokens travel to
//             rank d (one grouped send/recv, a fixed-size block per peer, so
//             no host synchronisation is needed to size it).
// The owner then sums its tokens' rows in ascending expert id, as on one GPU.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy a host
// framework may already have loaded), so the single-GPU library carries no
// NCCL dependency.
#include <dlfcn.h>
#include <time.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include <nccl.h>

#include "fw_kernels.h"

namespace fw {
namespace {

struct NcclApi {
  bool ok = false;
  char why[160] = {};
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
};

const NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (lib == nullptr) {
      std::snprintf(a.why, sizeof a.why, "libnccl.so.2 not loadable: %s", dlerror());
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
      if (fn == nullptr) all = false;
    };
    get(a.get_unique_id, "ncclGetUniqueId");
    get(a.comm_init_rank, "ncclCommInitRank");
    get(a.comm_destroy, "ncclCommDestroy");
    get(a.comm_abort, "ncclCommAbort");
    get(a.async_error, "ncclCommGetAsyncError");
    get(a.error_string, "ncclGetErrorString");
    get(a.all_gather, "ncclAllGather");
    get(a.send, "ncclSend");
    get(a.recv, "ncclRecv");
    get(a.group_start, "ncclGroupStart");
    get(a.group_end, "ncclGroupEnd");
    if (!all) {
      std::snprintf(a.why, sizeof a.why, "libnccl.so.2 lacks an entry point this library needs");
      return;
    }
    a.ok = true;
  });
  return a;
}

thread_local char g_msg[256];

const char* nccl_fail(const char* what, ncclResult_t r) {
  std::snprintf(g_msg, sizeof g_msg, "%s: %s", what, api().error_string(r));
  return g_msg;
}

}  // namespace

struct EpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool aborted = false;  // ncclCommAbort ran: every later call fails
};

const char* ep_unique_id(unsigned char out[128]) {
  const NcclApi& a = api();
  if (!a.ok) return a.why;
  ncclUniqueId id;
  const ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  static_assert(sizeof id.internal == 128, "NCCL unique id size");
  std::memcpy(out, id.internal, 128);
  return nullptr;
}

const char* ep_comm_init(int rank, int world, const unsigned char id_bytes[128], EpComm** out) {
  const NcclApi& a = api();
  if (!a.ok) return a.why;
  ncclUniqueId id;
  std::memcpy(id.internal, id_bytes, 128);
  EpComm* c = new EpComm();
  c->rank = rank;
  c->world = world;
  const ncclResult_t r = a.comm_init_rank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail("ncclCommInitRank", r);
  }
  *out = c;
  return nullptr;
}

// Teardown never waits on the peers (a peer may be gone): the communicator
// is aborted rather than destroyed, which releases it locally.
void ep_comm_destroy(EpComm* c) {
  if (c == nullptr) return;
  if (c->comm != nullptr && !c->aborted && api().ok) api().comm_abort(c->comm);
  delete c;
}

// Wait for `st` (the handle's forwards, NCCL kernels included) for at most
// `limit_ns`, watching the communicator's asynchronous error.  When a peer
// never joins a collective, NCCL's kernel keeps waiting for it: the
// communicator is then aborted, which ends that kernel, and every later
// forward on the handle fails.  Returns 0, 1 (timeout, aborted), 2 (NCCL
// error, aborted) or 3 (a CUDA error, in *cuda_err).
int ep_bounded_sync(EpComm* c, cudaStream_t st, unsigned long long limit_ns, cudaError_t* cuda_err) {
  const NcclApi& a = api();
  timespec t0;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) {
      *cuda_err = q;
      return 3;
    }
    if (c != nullptr && !c->aborted && a.ok) {
      ncclResult_t ae = ncclSuccess;
      if (a.async_error(c->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
        a.comm_abort(c->comm);
        c->aborted = true;
        return 2;
      }
    }
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    const unsigned long long el = static_cast<unsigned long long>(t.tv_sec - t0.tv_sec) * 1000000000ull +
                                  static_cast<unsigned long long>(t.tv_nsec) - static_cast<unsigned long long>(t0.tv_nsec);
    if (el > limit_ns) {
      if (c != nullptr && !c->aborted && a.ok) {
        a.comm_abort(c->comm);
        c->aborted = true;
      }
      return 1;
    }
    usleep(50);
  }
}

bool ep_comm_aborted(const EpComm* c) { return c != nullptr && c->aborted; }

const char* ep_dispatch(EpComm* c, const uint16_t* x, uint16_t* x_all, size_t x_elems, const int32_t* idx,
                        int32_t* idx_all, const uint16_t* score, uint16_t* score_all, size_t k_elems,
                        cudaStream_t st) {
  const NcclApi& a = api();
  ncclResult_t r = a.group_start();
  if (r != ncclSuccess) return nccl_fail("ncclGroupStart", r);
  ncclResult_t r1 = a.all_gather(x, x_all, x_elems, ncclBfloat16, c->comm, st);
  ncclResult_t r2 = a.all_gather(idx, idx_all, k_elems, ncclInt32, c->comm, st);
  ncclResult_t r3 = a.all_gather(score, score_all, k_elems, ncclBfloat16, c->comm, st);
  r = a.group_end();
  if (r1 != ncclSuccess) return nccl_fail("ncclAllGather (token rows)", r1);
  if (r2 != ncclSuccess) return nccl_fail("ncclAllGather (top-k ids)", r2);
  if (r3 != ncclSuccess) return nccl_fail("ncclAllGather (route weights)", r3);
  if (r != ncclSuccess) return nccl_fail("ncclGroupEnd", r);
  return nullptr;
}

const char* ep_combine_exchange(EpComm* c, const uint16_t* send, uint16_t* recv, size_t block_elems,
                                cudaStream_t st) {
  const NcclApi& a = api();
  ncclResult_t r = a.group_start();
  if (r != ncclSuccess) return nccl_fail("ncclGroupStart", r);
  ncclResult_t bad = ncclSuccess;
  for (int p = 0; p < c->world; ++p) {
    const ncclResult_t s1 = a.send(send + static_cast<size_t>(p) * block_elems, block_elems, ncclBfloat16, p,
                                   c->comm, st);
    const ncclResult_t s2 = a.recv(recv + static_cast<size_t>(p) * block_elems, block_elems, ncclBfloat16, p,
                                   c->comm, st);
    if (bad == ncclSuccess) bad = s1 != ncclSuccess ? s1 : s2;
  }
  r = a.group_end();
  if (bad != ncclSuccess) return nccl_fail("ncclSend / ncclRecv", bad);
  if (r != ncclSuccess) return nccl_fail("ncclGroupEnd", r);
  return nullptr;
}

const char* ep_exchange_rows(EpComm* c, const uint16_t* send, const int* rows_send, const int* off_send,
                             uint16_t* recv, const int* rows_recv, const int* off_recv, size_t row_elems,
                             cudaStream_t st) {
  const NcclApi& a = api();
  ncclResult_t r = a.group_start();
  if (r != ncclSuccess) return nccl_fail("ncclGroupStart", r);
  ncclResult_t bad = ncclSuccess;
  for (int p = 0; p < c->world; ++p) {
    ncclResult_t s1 = ncclSuccess, s2 = ncclSuccess;
    if (rows_send[p] > 0)
      s1 = a.send(send + static_cast<size_t>(off_send[p]) * row_elems, static_cast<size_t>(rows_send[p]) * row_elems,
                  ncclBfloat16, p, c->comm, st);
    if (rows_recv[p] > 0)
      s2 = a.recv(recv + static_cast<size_t>(off_recv[p]) * row_elems, static_cast<size_t>(rows_recv[p]) * row_elems,
                  ncclBfloat16, p, c->comm, st);
    if (bad == ncclSuccess) bad = s1 != ncclSuccess ? s1 : s2;
  }
  r = a.group_end();
  if (bad != ncclSuccess) return nccl_fail("ncclSend / ncclRecv", bad);
  if (r != ncclSuccess) return nccl_fail("ncclGroupEnd", r);
  return nullptr;
}

const char* ep_async_error(EpComm* c) {
  if (c == nullptr || !api().ok) return nullptr;
  ncclResult_t e = ncclSuccess;
  const ncclResult_t r = api().async_error(c->comm, &e);
  if (r != ncclSuccess) return nccl_fail("ncclCommGetAsyncError", r);
  if (e != ncclSuccess && e != ncclInProgress) return nccl_fail("NCCL communicator", e);
  return nullptr;
}

}  // namespace fw
