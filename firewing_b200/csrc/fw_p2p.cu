// fw_p2p.cu -- the expert-parallel exchange over NVLink peer memory.
//
// Rank r of N holds the experts e with e % N == r and brings its own tokens.
// Instead of collectives, every rank owns one exchange window (EpPeers in
// fw_kernels.h) that every other rank maps into its own address space, and
// the block's two exchange steps become plain loads and stores over NVLink:
//
//   publish   this rank copies its token rows, top-k ids and route weights
//             into its window, then sets its `pub` flag in every window;
//   dispatch  each rank waits (bounded) for every pub flag, reads every
//             rank's ids, and pulls each token row it needs ONCE (a token
//             selecting three of this rank's experts crosses NVLink once)
//             straight into its grouped GEMM input (prefill) or its gathered
//             rows (decode);
//   combine   the expert kernels' epilogues store each weighted row
//             straight into the owner's receive area (row t*K + k), so the
//             transfer overlaps the GEMM tile by tile; the last CTA of the
//             expert kernel sets this rank's `done` flag in every window,
//             and the owner's combine waits (bounded) for all of them before
//             it sums its tokens' rows in ascending expert id.
//
// No host synchronisation sizes anything: positions follow from the ids.
// Windows are never reused before every reader is done with them (the flags
// of forward s+1 are set only after the combine of forward s).
//
// Memory: each window is a cuMem allocation exported as a POSIX file
// descriptor; the descriptors travel between the ranks' processes over
// abstract Unix datagram sockets (SCM_RIGHTS) named after the communicator
// id, and every rank maps every window.  Physical memory is reference
// counted by its handles, so a window stays valid for the ranks that mapped
// it even after its owner exits: a rank that stops taking part makes the
// others' bounded waits expire (FW_ETIMEOUT), never a fault.
//
// No load here or in the kernels that read peer windows uses TMA, let alone
// cluster multicast: peer data moves with plain 16-byte loads and stores.
#include <fcntl.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <time.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

// ---- driver entry points (no link-time dependency on libcuda) -----------------
struct VmmApi {
  bool ok = false;
  PFN_cuMemGetAllocationGranularity_v10020 granularity = nullptr;
  PFN_cuMemCreate_v10020 create = nullptr;
  PFN_cuMemRelease_v10020 release = nullptr;
  PFN_cuMemExportToShareableHandle_v10020 export_fd = nullptr;
  PFN_cuMemImportFromShareableHandle_v10020 import_fd = nullptr;
  PFN_cuMemAddressReserve_v10020 reserve = nullptr;
  PFN_cuMemAddressFree_v10020 address_free = nullptr;
  PFN_cuMemMap_v10020 map = nullptr;
  PFN_cuMemUnmap_v10020 unmap = nullptr;
  PFN_cuMemSetAccess_v10020 set_access = nullptr;
};

const VmmApi& vmm() {
  static VmmApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        all = false;
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(p);
    };
    get(a.granularity, "cuMemGetAllocationGranularity");
    get(a.create, "cuMemCreate");
    get(a.release, "cuMemRelease");
    get(a.export_fd, "cuMemExportToShareableHandle");
    get(a.import_fd, "cuMemImportFromShareableHandle");
    get(a.reserve, "cuMemAddressReserve");
    get(a.address_free, "cuMemAddressFree");
    get(a.map, "cuMemMap");
    get(a.unmap, "cuMemUnmap");
    get(a.set_access, "cuMemSetAccess");
    a.ok = all;
  });
  return a;
}

thread_local char g_msg[256];

const char* msgf(const char* fmt, long a = 0, long b = 0) {
  std::snprintf(g_msg, sizeof g_msg, fmt, a, b);
  return g_msg;
}

uint64_t now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return static_cast<uint64_t>(ts.tv_sec) * 1000u + static_cast<uint64_t>(ts.tv_nsec) / 1000000u;
}

// Abstract socket address of `rank` in the communicator named by `tag`.
socklen_t socket_name(sockaddr_un* a, uint64_t tag, int rank) {
  std::memset(a, 0, sizeof *a);
  a->sun_family = AF_UNIX;
  const int n = std::snprintf(a->sun_path + 1, sizeof a->sun_path - 1, "fwmoe-ep-%016llx-%d",
                              static_cast<unsigned long long>(tag), rank);
  return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
}

struct FdMsg {
  uint32_t magic;
  int32_t rank;
  uint64_t tag;
  uint64_t bytes;
};
constexpr uint32_t kFdMagic = 0x46574550u;  // "FWEP"

// Send `fd` to every peer's socket and receive one descriptor from each
// peer, within `deadline_ms`.  Peers bind before they send, so a send to a
// socket that does not exist yet is retried until the deadline.
const char* exchange_fds(int sock, uint64_t tag, int rank, int world, int fd, uint64_t bytes, int* peer_fd,
                         uint64_t deadline_ms) {
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    sockaddr_un to;
    const socklen_t len = socket_name(&to, tag, p);
    FdMsg m{kFdMagic, rank, tag, bytes};
    for (;;) {
      iovec io{&m, sizeof m};
      char ctl[CMSG_SPACE(sizeof(int))];
      std::memset(ctl, 0, sizeof ctl);
      msghdr h{};
      h.msg_name = &to;
      h.msg_namelen = len;
      h.msg_iov = &io;
      h.msg_iovlen = 1;
      h.msg_control = ctl;
      h.msg_controllen = sizeof ctl;
      cmsghdr* c = CMSG_FIRSTHDR(&h);
      c->cmsg_level = SOL_SOCKET;
      c->cmsg_type = SCM_RIGHTS;
      c->cmsg_len = CMSG_LEN(sizeof(int));
      std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
      if (sendmsg(sock, &h, 0) == static_cast<ssize_t>(sizeof m)) break;
      if (errno != ECONNREFUSED && errno != ENOENT && errno != EAGAIN && errno != EINTR)
        return msgf("expert parallelism: sending the window to rank %ld failed (errno %ld)", p, errno);
      if (now_ms() > deadline_ms) return msgf("expert parallelism: rank %ld did not open its socket in time", p);
      usleep(1000);
    }
  }
  for (int got = 0; got < world - 1;) {
    const uint64_t t = now_ms();
    if (t > deadline_ms) return msgf("expert parallelism: received %ld of %ld peer windows in time", got, world - 1);
    pollfd pf{sock, POLLIN, 0};
    const int pr = poll(&pf, 1, static_cast<int>(deadline_ms - t));
    if (pr < 0 && errno == EINTR) continue;
    if (pr <= 0) continue;
    FdMsg m{};
    iovec io{&m, sizeof m};
    char ctl[CMSG_SPACE(sizeof(int))];
    msghdr h{};
    h.msg_iov = &io;
    h.msg_iovlen = 1;
    h.msg_control = ctl;
    h.msg_controllen = sizeof ctl;
    const ssize_t n = recvmsg(sock, &h, MSG_CMSG_CLOEXEC);
    if (n < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      return msgf("expert parallelism: receiving a peer window failed (errno %ld)", errno);
    }
    cmsghdr* c = CMSG_FIRSTHDR(&h);
    int rfd = -1;
    if (c != nullptr && c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) std::memcpy(&rfd, CMSG_DATA(c), sizeof(int));
    if (n != static_cast<ssize_t>(sizeof m) || m.magic != kFdMagic || m.tag != tag || m.rank < 0 || m.rank >= world ||
        m.rank == rank || rfd < 0 || peer_fd[m.rank] >= 0 || m.bytes != bytes) {
      if (rfd >= 0) close(rfd);
      return "expert parallelism: a peer sent a window of another communicator or shape";
    }
    peer_fd[m.rank] = rfd;
    ++got;
  }
  return nullptr;
}

}  // namespace

struct P2pComm {
  int device = 0, rank = 0, world = 1;
  size_t win_bytes = 0;                 // per window, a multiple of the allocation granularity
  CUdeviceptr base = 0;                 // world consecutive windows
  bool mapped[kEpMaxWorld] = {};
  CUmemGenericAllocationHandle own = 0;
  bool own_valid = false;
  long long off_x = 0, off_idx = 0, off_score = 0, off_recv = 0;
  int H = 0, K = 0, max_tokens = 0;
  int* tickets = nullptr;               // [2] signalling-kernel counters
};

void p2p_destroy(P2pComm* c) {
  if (c == nullptr) return;
  const VmmApi& a = vmm();
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  if (a.ok) {
    for (int r = 0; r < c->world; ++r)
      if (c->mapped[r]) a.unmap(c->base + static_cast<CUdeviceptr>(r) * c->win_bytes, c->win_bytes);
    if (c->own_valid) a.release(c->own);
    if (c->base != 0) a.address_free(c->base, c->win_bytes * c->world);
  }
  if (c->tickets != nullptr) cudaFree(c->tickets);
  delete c;
}

size_t p2p_window_bytes(const P2pComm* c) { return c == nullptr ? 0 : c->win_bytes; }

const char* p2p_init(int device, int rank, int world, const unsigned char id[128], int max_tokens, int H, int K,
                     P2pComm** out) {
  *out = nullptr;
  const VmmApi& a = vmm();
  if (!a.ok) return "expert parallelism over peer memory: the driver lacks the cuMem entry points";
  if (world < 2 || world > kEpMaxWorld) return "expert parallelism over peer memory: world must be 2..8";
  auto* c = new P2pComm();
  c->device = device;
  c->rank = rank;
  c->world = world;
  c->H = H;
  c->K = K;
  c->max_tokens = max_tokens;
  const char* m = nullptr;
  int sock = -1;
  int my_fd = -1;
  int peer_fd[kEpMaxWorld];
  for (int& f : peer_fd) f = -1;
  do {
    // Window layout (see EpPeers).
    auto align = [](long long v) { return (v + 255) & ~255LL; };
    const long long M = max_tokens;
    c->off_x = 256;
    c->off_idx = align(c->off_x + M * H * 2);
    c->off_score = align(c->off_idx + M * K * 4);
    c->off_recv = align(c->off_score + M * K * 2);
    const size_t need = static_cast<size_t>(align(c->off_recv + M * K * H * 2));
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    if (a.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || gran == 0) {
      m = "expert parallelism: cuMemGetAllocationGranularity failed";
      break;
    }
    c->win_bytes = (need + gran - 1) / gran * gran;
    if (a.reserve(&c->base, c->win_bytes * world, gran, 0, 0) != CUDA_SUCCESS) {
      m = "expert parallelism: reserving the windows' address range failed";
      break;
    }
    if (a.create(&c->own, c->win_bytes, &prop, 0) != CUDA_SUCCESS) {
      m = "expert parallelism: cuMemCreate of the exchange window failed (out of memory?)";
      break;
    }
    c->own_valid = true;
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    const CUdeviceptr mine = c->base + static_cast<CUdeviceptr>(rank) * c->win_bytes;
    if (a.map(mine, c->win_bytes, 0, c->own, 0) != CUDA_SUCCESS ||
        a.set_access(mine, c->win_bytes, &acc, 1) != CUDA_SUCCESS) {
      m = "expert parallelism: mapping the own window failed";
      break;
    }
    c->mapped[rank] = true;
    // Flags at zero before any peer can map the window.
    if (cudaMemset(reinterpret_cast<void*>(mine), 0, 256) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
      m = "expert parallelism: clearing the window's flags failed";
      break;
    }
    if (cudaMalloc(&c->tickets, 2 * sizeof(int)) != cudaSuccess ||
        cudaMemset(c->tickets, 0, 2 * sizeof(int)) != cudaSuccess) {
      m = "expert parallelism: ticket allocation failed";
      break;
    }
    if (a.export_fd(&my_fd, c->own, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS || my_fd < 0) {
      m = "expert parallelism: exporting the window as a file descriptor failed";
      break;
    }
    // The communicator's name: FNV-1a of its 128-byte id.
    uint64_t tag = 1469598103934665603ull;
    for (int i = 0; i < 128; ++i) tag = (tag ^ id[i]) * 1099511628211ull;
    sock = socket(AF_UNIX, SOCK_DGRAM | SOCK_CLOEXEC | SOCK_NONBLOCK, 0);
    sockaddr_un me;
    const socklen_t len = socket_name(&me, tag, rank);
    if (sock < 0 || bind(sock, reinterpret_cast<sockaddr*>(&me), len) != 0) {
      m = msgf("expert parallelism: binding the rank's socket failed (errno %ld)", errno);
      break;
    }
    m = exchange_fds(sock, tag, rank, world, my_fd, c->win_bytes, peer_fd, now_ms() + 120000);
    if (m != nullptr) break;
    for (int p = 0; p < world && m == nullptr; ++p) {
      if (p == rank) continue;
      CUmemGenericAllocationHandle h = 0;
      const CUdeviceptr at = c->base + static_cast<CUdeviceptr>(p) * c->win_bytes;
      if (a.import_fd(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(peer_fd[p])),
                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) != CUDA_SUCCESS) {
        m = msgf("expert parallelism: importing rank %ld's window failed", p);
        break;
      }
      // The mapping keeps the peer's memory alive; the handle itself is not needed.
      const bool ok = a.map(at, c->win_bytes, 0, h, 0) == CUDA_SUCCESS;
      a.release(h);
      if (!ok || a.set_access(at, c->win_bytes, &acc, 1) != CUDA_SUCCESS) {
        if (ok) a.unmap(at, c->win_bytes);
        m = msgf("expert parallelism: mapping rank %ld's window failed (no peer access over NVLink?)", p);
        break;
      }
      c->mapped[p] = true;
    }
  } while (false);
  if (sock >= 0) close(sock);
  if (my_fd >= 0) close(my_fd);
  for (int f : peer_fd)
    if (f >= 0) close(f);
  if (m != nullptr) {
    p2p_destroy(c);
    return m;
  }
  *out = c;
  return nullptr;
}

EpPeers p2p_peers(const P2pComm* c, int t_local, unsigned seq, unsigned long long wait_ns) {
  EpPeers p;
  for (int r = 0; r < c->world; ++r)
    p.win[r] = reinterpret_cast<unsigned char*>(c->base + static_cast<CUdeviceptr>(r) * c->win_bytes);
  p.rank = c->rank;
  p.world = c->world;
  p.t_local = t_local;
  p.K = c->K;
  p.H = c->H;
  p.off_x = c->off_x;
  p.off_idx = c->off_idx;
  p.off_score = c->off_score;
  p.off_recv = c->off_recv;
  p.seq = seq;
  p.wait_ns = wait_ns;
  p.ticket = c->tickets;
  return p;
}

uint16_t* p2p_recv(const P2pComm* c) {
  return reinterpret_cast<uint16_t*>(c->base + static_cast<CUdeviceptr>(c->rank) * c->win_bytes + c->off_recv);
}

// ---- kernels ---------------------------------------------------------------

namespace {

// Copy this rank's token rows, ids and route weights into its window, then
// (last CTA) set its pub flag in every window.
__global__ void __launch_bounds__(256) k_ep_publish(EpPeers p, const uint16_t* x, const int32_t* idx,
                                                    const uint16_t* score, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long nthreads = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nx = static_cast<long long>(p.t_local) * p.H / 8;  // 16-byte chunks
  uint4* dx = reinterpret_cast<uint4*>(p.win[p.rank] + p.off_x);
  const uint4* sx = reinterpret_cast<const uint4*>(x);
  for (long long i = tid; i < nx; i += nthreads) dx[i] = sx[i];
  const long long nk = static_cast<long long>(p.t_local) * p.K;
  int32_t* di = reinterpret_cast<int32_t*>(p.win[p.rank] + p.off_idx);
  uint16_t* ds = reinterpret_cast<uint16_t*>(p.win[p.rank] + p.off_score);
  for (long long i = tid; i < nk; i += nthreads) {
    di[i] = idx[i];
    ds[i] = score[i];
  }
  ep_signal(p, kEpFlagPub, p.ticket + 0, err);
}

// Decode widths: after every rank has published, warp g brings token g of
// the gathered index space (rank g / t_local): its ids and route weights
// into idx_all / score_all, and its row into x_all when one of its experts
// is this rank's.
__global__ void __launch_bounds__(256) k_ep_pull(EpPeers p, int E, int32_t* idx_all, uint16_t* score_all,
                                                 uint16_t* x_all, int* err) {
  __shared__ int s_ok;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) s_ok = ep_wait_flags(p, kEpFlagPub, err) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int lane = threadIdx.x & 31;
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (g >= p.world * p.t_local) return;
  const int src = g / p.t_local, t = g - src * p.t_local;
  const int32_t* ri = reinterpret_cast<const int32_t*>(p.win[src] + p.off_idx) + static_cast<size_t>(t) * p.K;
  const uint16_t* rs = reinterpret_cast<const uint16_t*>(p.win[src] + p.off_score) + static_cast<size_t>(t) * p.K;
  bool local = false;
  for (int k = lane; k < p.K; k += 32) {
    const int e = ri[k];
    if (e < 0 || e >= E) {
      set_error(err, kErrBadIndex);
      continue;
    }
    idx_all[static_cast<size_t>(g) * p.K + k] = e;
    score_all[static_cast<size_t>(g) * p.K + k] = rs[k];
    local |= e % p.world == p.rank;
  }
  if (!__any_sync(0xffffffffu, local)) return;
  const uint4* sx = reinterpret_cast<const uint4*>(p.win[src] + p.off_x) + static_cast<size_t>(t) * (p.H / 8);
  uint4* dx = reinterpret_cast<uint4*>(x_all) + static_cast<size_t>(g) * (p.H / 8);
  for (int c = lane; c < p.H / 8; c += 32) dx[c] = sx[c];
}

// Prefill widths, step 1: after every rank has published, every (token, k)
// of the gathered index space: its id and route weight into idx_all /
// score_all, and the pair counts of this rank's experts (bank e / world).
__global__ void __launch_bounds__(256) k_ep_ids(EpPeers p, int E, int32_t* idx_all, uint16_t* score_all, int* count,
                                                int* err) {
  __shared__ int s_ok;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) s_ok = ep_wait_flags(p, kEpFlagPub, err) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const long long n = static_cast<long long>(p.world) * p.t_local * p.K;
  const long long per_rank = static_cast<long long>(p.t_local) * p.K;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int src = static_cast<int>(i / per_rank);
    const long long j = i - src * per_rank;
    const int e = reinterpret_cast<const int32_t*>(p.win[src] + p.off_idx)[j];
    if (e < 0 || e >= E) {
      set_error(err, kErrBadIndex);
      idx_all[i] = 0;
      continue;
    }
    idx_all[i] = e;
    score_all[i] = reinterpret_cast<const uint16_t*>(p.win[src] + p.off_score)[j];
    if (e % p.world == p.rank) atomicAdd(&count[e / p.world], 1);
  }
}

// Prefill widths, step 2 (after the pair offsets): warp g takes token g of
// the gathered index space, gives each of its pairs with one of this rank's
// experts a slot in that expert's group, and copies the token's row once
// from its owner's window into every slot's row of the grouped input xg
// (K-blocked, [H/64][xg_rows][64]).  Slots are counted per CTA in shared
// memory and each expert's range reserved with one global atomic per CTA
// (a hot expert draws pairs from every rank's tokens).
__global__ void __launch_bounds__(256) k_ep_scatter(EpPeers p, int banks, const int32_t* idx_all, const int* offset,
                                                    int* fill, int32_t* pair_tk, uint16_t* xg, long long xg_rows,
                                                    int* err) {
  extern __shared__ int s_cnt[];  // [banks]: this CTA's pairs per bank, then their base in the group
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_bad;
  const int lane = threadIdx.x & 31;
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const bool live = g < p.world * p.t_local;
  if (threadIdx.x == 0) s_bad = ld_volatile_int(err);
  for (int i = threadIdx.x; i < banks; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  if (s_bad != 0) return;  // one read per CTA: the whole CTA leaves together
  int bank = -1, lr = 0;
  if (live && lane < p.K) {
    const int e = idx_all[static_cast<size_t>(g) * p.K + lane];
    if (e % p.world == p.rank) {
      bank = e / p.world;
      lr = atomicAdd(&s_cnt[bank], 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < banks; i += blockDim.x) {
    const int c = s_cnt[i];
    if (c > 0) s_cnt[i] = atomicAdd(&fill[i], c);
  }
  __syncthreads();
  int slot = -1;
  if (bank >= 0) {
    slot = offset[bank] + s_cnt[bank] + lr;
    pair_tk[slot] = g * p.K + lane;
  }
  const unsigned have = __ballot_sync(0xffffffffu, slot >= 0);
  if (!live || have == 0) return;
  const int src = g / p.t_local, t = g - src * p.t_local;
  const uint4* sx = reinterpret_cast<const uint4*>(p.win[src] + p.off_x) + static_cast<size_t>(t) * (p.H / 8);
  const int nch = p.H / 8;
  // Four chunks in flight per lane; each goes to every slot of the token.
  for (int c0 = lane; c0 < nch; c0 += 4 * 32) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c0 + 32 * u < nch) v[u] = sx[c0 + 32 * u];
    unsigned rest = have;
    while (rest != 0) {
      const int src_lane = __ffs(rest) - 1;
      rest &= rest - 1;
      const long long row = __shfl_sync(0xffffffffu, slot, src_lane);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c < nch)
          *reinterpret_cast<uint4*>(xg + ((static_cast<long long>(c >> 3) * xg_rows + row) * 64 + (c & 7) * 8)) = v[u];
      }
    }
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

int grid_for(long long work, int per_block, int cap) {
  const long long b = (work + per_block - 1) / per_block;
  return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

cudaError_t launch_ep_publish(const EpPeers& p, const uint16_t* x, const int32_t* idx, const uint16_t* score, int* err,
                              cudaStream_t st) {
  const long long chunks = static_cast<long long>(p.t_local) * p.H / 8;
  return launch_pdl(k_ep_publish, dim3(grid_for(chunks, 256 * 4, 4 * 148)), dim3(256), st, p, x, idx, score, err);
}

cudaError_t launch_ep_pull(const EpPeers& p, int E, int32_t* idx_all, uint16_t* score_all, uint16_t* x_all, int* err,
                           cudaStream_t st) {
  const int tokens = p.world * p.t_local;
  return launch_pdl(k_ep_pull, dim3((tokens + 7) / 8), dim3(256), st, p, E, idx_all, score_all, x_all, err);
}

cudaError_t launch_ep_ids(const EpPeers& p, int E, int32_t* idx_all, uint16_t* score_all, int* count, int* err,
                          cudaStream_t st) {
  const long long n = static_cast<long long>(p.world) * p.t_local * p.K;
  return launch_pdl(k_ep_ids, dim3(grid_for(n, 256, 8 * 148)), dim3(256), st, p, E, idx_all, score_all, count, err);
}

cudaError_t launch_ep_scatter(const EpPeers& p, int banks, const int32_t* idx_all, const int* offset, int* fill,
                              int32_t* pair_tk, uint16_t* xg, long long xg_rows, int* err, cudaStream_t st) {
  const int tokens = p.world * p.t_local;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((tokens + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = sizeof(int) * static_cast<size_t>(banks);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_ep_scatter, p, banks, idx_all, offset, fill, pair_tk, xg, xg_rows, err);
}

}  // namespace fw
