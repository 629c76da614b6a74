// ep.cu -- expert parallelism across the GPUs of one node (one process per GPU).
//
// No counterpart in the reference, which runs on one device.  Rank r owns
// experts [r*E/N, (r+1)*E/N) and routes its own tokens.  Per forward (epoch e,
// the same count on every rank):
//
//   1. count exchange   per-expert position counts, E/N ints to every peer
//                       (NCCL, non-blocking communicator, host deadline); the
//                       host learns how many positions it will run
//   2. dispatch         a kernel writes each token's activation row ONCE per
//                       destination rank (not once per expert) straight into
//                       that rank's receive buffer over NVLink (peer stores),
//                       with a 16-byte descriptor (token, local expert of each
//                       of its k ranks); the last CTA releases flag[s] = e on
//                       every destination
//   3. local grouping   one CTA waits (bounded) for every source's flag and
//                       orders the received rows' (row, expert) positions by
//                       local expert, then source
//   4. experts          the single-GPU expert kernels on the received rows;
//                       the block-scaled down GEMM stores each output row
//                       straight into its source rank's return slot t*k + r
//                       (peer stores from the epilogue, overlapping the math);
//                       the other kernels' rows go by a copy kernel
//   5. return signal    after the down stage, flag_ret[r] = e on every rank
//   6. combine          waits (bounded) for every rank's return flag, then the
//                       single-GPU combine over the return slots: the same
//                       rank order, so the sums are those of one GPU
//
// The receive buffers, descriptors, flags and return slots of every rank are
// one device allocation whose CUDA IPC handle is exchanged at create, so each
// rank holds the others' addresses.  Source s owns rows [s*Tc, (s+1)*Tc) of a
// destination's receive buffer (Tc = the largest max_tokens of the ranks), so
// no offsets need agreeing.  Buffers are reused by the next forward only after
// the combine of this one, which waits for every rank's return, which follows
// that rank's last read of the receive buffer: single buffers suffice.
//
// Failure handling: every NCCL call runs on a non-blocking communicator and
// the host polls it against a deadline (ep_timeout_ms of the descriptor,
// default 60 s), aborting the communicator when the deadline passes or NCCL
// reports an asynchronous error; every device-side flag wait is bounded by the
// same time and records GB_ERR_TIMEOUT in the error word.  A handle whose
// communicator was aborted refuses further forwards.  A peer that leaves
// between forwards is caught by the count exchange, before any peer store.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, the copy PyTorch has
// already loaded when there is one), so single-GPU use needs no NCCL.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "moe_internal.h"
#include "ptx.cuh"

namespace gb {

namespace {

constexpr int kMaxRanks = 8;  // one NVSwitch node

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

int load_nccl() {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl.lib) return GB_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return set_error(GB_ERR_NCCL, "cannot load NCCL (libnccl.so.2): %s", dlerror());
  NcclApi a;
  a.lib = h;
#define GB_SYM(field, name)                                                         \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));                     \
  if (!a.field) return set_error(GB_ERR_NCCL, "NCCL symbol %s not found", name);
  GB_SYM(GetUniqueId, "ncclGetUniqueId")
  GB_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
  GB_SYM(CommFinalize, "ncclCommFinalize")
  GB_SYM(CommDestroy, "ncclCommDestroy")
  GB_SYM(CommAbort, "ncclCommAbort")
  GB_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
  GB_SYM(GroupStart, "ncclGroupStart")
  GB_SYM(GroupEnd, "ncclGroupEnd")
  GB_SYM(Send, "ncclSend")
  GB_SYM(Recv, "ncclRecv")
  GB_SYM(AllGather, "ncclAllGather")
  GB_SYM(AllReduce, "ncclAllReduce")
  GB_SYM(GetErrorString, "ncclGetErrorString")
#undef GB_SYM
  g_nccl = a;
  return GB_OK;
}

int nccl_err(ncclResult_t r, const char* what) {
  return set_error(GB_ERR_NCCL, "%s: %s", what,
                   g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error");
}

#define GB_CU(call, what)                                                                   \
  do {                                                                                      \
    cudaError_t _e = (call);                                                                \
    if (_e != cudaSuccess)                                                                  \
      return set_error(GB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e));               \
  } while (0)

}  // namespace

// Rows of every rank, as seen from this one (peer addresses from CUDA IPC;
// this rank's own entry is its local address).
struct EpPeers {
  float* recv_x[kMaxRanks];  // [N src][Tc][H] rows sent to that rank
  int4* desc[kMaxRanks];     // [N src][Tc] {token, local expert of ranks 0-3, of 4-7, 0}
  int* rows[kMaxRanks];      // [N src] rows each source sent
  int* flags[kMaxRanks];     // [2][N src]: dispatch epoch, return epoch
  float* y_back[kMaxRanks];  // [Tc * k][H] expert outputs for that rank's tokens
};

struct Ep {
  ncclComm_t comm = nullptr;
  bool broken = false;         // communicator aborted: no further forwards
  int rank = 0, size = 1, e_per = 0;
  int64_t tc = 0;              // receive rows per source (largest max_tokens)
  int64_t timeout_ms = 60000;  // host and device wait limit
  int epoch = 0;
  void* sym = nullptr;         // this rank's shared allocation
  size_t sym_bytes = 0;
  void* peer_base[kMaxRanks] = {};  // opened IPC mappings (null for this rank)
  EpPeers peers{};
  int32_t* cnt_recv = nullptr;  // [size][e_per] positions from each source per local expert
  int32_t* counts2 = nullptr;   // [E]
  int32_t* offsets2 = nullptr;  // [E+1]
  int32_t* active2 = nullptr;   // [E]
  int32_t* meta2 = nullptr;     // [4]
  int32_t* slot = nullptr;      // [Tc][size] row slot of token t at each destination, or -1
  int32_t* nrows = nullptr;     // [size] rows this rank sends to each destination
  unsigned* tickets = nullptr;  // [2] last-CTA tickets of the dispatch and return kernels
  int32_t* host = nullptr;      // mapped pinned: [max(E, 2)] received counts (or one int64)
  int32_t* host_dev = nullptr;  // its device address
  int32_t* perm2 = nullptr;     // [r_cap] received row of each position
  int64_t* ret2 = nullptr;      // [r_cap] (source rank << 32) | return slot of each position
  int64_t r_cap = 0;
  ExpertBufs eb;                // r_cap positions; y by position
};

namespace {

using Clock = std::chrono::steady_clock;

// Aborts the communicator (cancelling NCCL work stuck on a lost peer) and
// marks the handle unusable.
void abort_comm(Ep* ep) {
  if (ep->comm && g_nccl.CommAbort) g_nccl.CommAbort(ep->comm);
  ep->comm = nullptr;
  ep->broken = true;
}

// Completes a non-blocking NCCL call: polls the communicator until it leaves
// ncclInProgress, within the handle's deadline.
int nccl_settle(Ep* ep, ncclResult_t r, const char* what) {
  if (r != ncclSuccess && r != ncclInProgress) {
    abort_comm(ep);
    return nccl_err(r, what);
  }
  const auto deadline = Clock::now() + std::chrono::milliseconds(ep->timeout_ms);
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = g_nccl.CommGetAsyncError(ep->comm, &st);
    if (q != ncclSuccess) st = q;
    if (st == ncclSuccess) return GB_OK;
    if (st != ncclInProgress) {
      abort_comm(ep);
      return nccl_err(st, what);
    }
    if (Clock::now() > deadline) {
      abort_comm(ep);
      return set_error(GB_ERR_TIMEOUT, "%s: NCCL did not finish within %lld ms", what,
                       (long long)ep->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Waits for `st` (which holds NCCL work) within the deadline, watching the
// communicator for asynchronous errors.  On failure the communicator is
// aborted, which ends its kernels, and the stream is given a bounded time to
// drain.
int stream_settle(Ep* ep, cudaStream_t st, const char* what) {
  const auto deadline = Clock::now() + std::chrono::milliseconds(ep->timeout_ms);
  int rc = GB_OK;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return GB_OK;
    if (q != cudaErrorNotReady) return set_error(GB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(q));
    ncclResult_t as = ncclSuccess;
    if (ep->comm && g_nccl.CommGetAsyncError(ep->comm, &as) == ncclSuccess &&
        as != ncclSuccess && as != ncclInProgress) {
      abort_comm(ep);
      rc = nccl_err(as, what);
      break;
    }
    if (Clock::now() > deadline) {
      abort_comm(ep);
      rc = set_error(GB_ERR_TIMEOUT, "%s: a peer did not answer within %lld ms", what,
                     (long long)ep->timeout_ms);
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
  const auto drain = Clock::now() + std::chrono::milliseconds(ep->timeout_ms);
  while (cudaStreamQuery(st) == cudaErrorNotReady && Clock::now() < drain)
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  return rc;
}

}  // namespace

namespace {

// ---- device side ----------------------------------------------------------

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag >= epoch (flags only grow); false on timeout.
__device__ __forceinline__ bool wait_epoch(const int* flag, int epoch, uint64_t timeout_ns) {
  if (ld_acquire_sys(flag) - epoch >= 0) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flag) - epoch < 0) {
    if (globaltimer() - t0 > timeout_ns) return false;
    __nanosleep(200);
  }
  return true;
}

// Destination d's row slot of every token: the tokens with at least one of
// their k experts on rank d, numbered in token order.  One CTA per
// destination, a block scan per 1024 tokens.
__global__ void __launch_bounds__(1024)
    ep_slots_kernel(const int32_t* __restrict__ idx, int T, int K, int e_per, int N,
                    int32_t* __restrict__ slot, int32_t* __restrict__ nrows) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  const int d = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    int has = 0;
    if (t < T)
      for (int r = 0; r < K; ++r) {
        const int e = idx[(int64_t)t * K + r];
        has |= e >= 0 && e / e_per == d;
      }
    int incl = has;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
      const int v = __shfl_up_sync(kFullMask, incl, s);
      if (lane >= s) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int v = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int s = 1; s < 32; s <<= 1) {
        const int u = __shfl_up_sync(kFullMask, v, s);
        if (lane >= s) v += u;
      }
      if (lane < nw) warp_tot[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    const int excl = incl - has + (warp ? warp_tot[warp - 1] : 0);
    if (t < T) slot[(int64_t)t * N + d] = has ? base + excl : -1;
    __syncthreads();
    if (threadIdx.x == 0) base += warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) nrows[d] = base;
}

// One CTA per token: its row, loaded once, stored into every destination
// rank that holds one of its experts (peer stores over NVLink), with the
// descriptor.  The last CTA to finish publishes the row counts and the
// dispatch flags.  Needs H % 4 == 0 and H <= 4096.
constexpr int kDispatchThreads = 128;

__global__ void __launch_bounds__(kDispatchThreads)
    ep_dispatch_kernel(const float* __restrict__ x, int T, int H, int K, int e_per,
                       const int32_t* __restrict__ idx, const int32_t* __restrict__ slot,
                       const int32_t* __restrict__ nrows, int me, int N, int64_t tc, EpPeers p,
                       int epoch, unsigned* __restrict__ ticket) {
  __shared__ bool last;
  const int t = blockIdx.x;
  if (t < T) {
    constexpr int kPer = 4096 / 4 / kDispatchThreads;
    const int n4 = H / 4;
    const float4* src = reinterpret_cast<const float4*>(x + (int64_t)t * H);
    float4 v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = threadIdx.x + i * kDispatchThreads;
      if (c < n4) v[i] = src[c];
    }
    int e[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) e[r] = r < K ? idx[(int64_t)t * K + r] : -1;
    for (int d = 0; d < N; ++d) {
      const int j = slot[(int64_t)t * N + d];
      if (j < 0) continue;
      const int64_t row = (int64_t)me * tc + j;
      float4* dst = reinterpret_cast<float4*>(p.recv_x[d] + row * H);
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * kDispatchThreads;
        if (c < n4) dst[c] = v[i];
      }
      if (threadIdx.x == 0) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint32_t le = (e[r] >= 0 && e[r] / e_per == d) ? (uint32_t)(e[r] - d * e_per) : 0xFFu;
          if (r < 4) lo |= le << (8 * r); else hi |= le << (8 * (r - 4));
        }
        p.desc[d][row] = make_int4(t, (int)lo, (int)hi, 0);
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  if (threadIdx.x < N) {
    const int d = threadIdx.x;
    p.rows[d][me] = nrows[d];
    __threadfence_system();
    st_release_sys(p.flags[d] + me, epoch);
  }
  if (threadIdx.x == 0) *ticket = 0;  // for the next forward
}

// Grouped view of the received rows: waits (bounded) for every source's
// dispatch flag, then places each (row, rank) entry whose expert is local at
// its position (local expert ascending, then source ascending; the order
// inside a (source, expert) run does not change any result).  One CTA.
__global__ void __launch_bounds__(1024)
    ep_plan_kernel(const int* __restrict__ flags, int epoch, uint64_t timeout_ns,
                   const int* __restrict__ rows, const int4* __restrict__ desc, int64_t tc,
                   const int32_t* __restrict__ cnt, int N, int e_per, int e_begin, int E, int K,
                   int64_t r_cap, int32_t* __restrict__ counts2, int32_t* __restrict__ offsets2,
                   int32_t* __restrict__ active2, int32_t* __restrict__ meta2,
                   int32_t* __restrict__ perm2, int64_t* __restrict__ ret2) {
  extern __shared__ int sh[];
  int* fill = sh;                     // [N * e_per]
  int* dst_off = fill + N * e_per;    // [N * e_per]
  int* cnt_s = dst_off + N * e_per;   // [N * e_per]
  __shared__ int ok, nrow[kMaxRanks];
  if (threadIdx.x == 0) ok = 1;
  for (int i = threadIdx.x; i < N * e_per; i += blockDim.x) {
    fill[i] = 0;
    cnt_s[i] = cnt[i];
  }
  // every position the host sized launches for points at a valid row and no
  // slot, whatever happens below (kernels after this one follow perm2)
  for (int64_t i = threadIdx.x; i < r_cap; i += blockDim.x) {
    perm2[i] = 0;
    ret2[i] = -1;
  }
  __syncthreads();
  if (threadIdx.x < N) {
    const int s = threadIdx.x;
    if (!wait_epoch(flags + s, epoch, timeout_ns)) {
      atomicAnd(&ok, 0);
      nrow[s] = 0;
    } else {
      nrow[s] = *reinterpret_cast<const volatile int*>(rows + s);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int pos = 0, nact = 0;
    for (int g = 0; g < E; ++g) {
      offsets2[g] = pos;
      const int e = g - e_begin;
      int n = 0;
      if (ok && e >= 0 && e < e_per) {
        for (int s = 0; s < N; ++s) {
          dst_off[s * e_per + e] = pos + n;
          n += cnt_s[s * e_per + e];
        }
        if (n > 0) active2[nact++] = g;
      }
      counts2[g] = n;
      pos += n;
    }
    offsets2[E] = pos;
    meta2[0] = nact;
    if (!ok) atomicOr(meta2 + 1, 2);  // a dispatch wait timed out: nothing runs
    if (pos > r_cap) {                // counts beyond the buffers: nothing runs
      atomicOr(meta2 + 1, 1);
      for (int g = 0; g <= E; ++g) offsets2[g] = 0;
      for (int g = 0; g < E; ++g) counts2[g] = 0;
      meta2[0] = 0;
      ok = 0;
    }
  }
  __syncthreads();
  if (!ok) return;
  for (int s = 0; s < N; ++s) {
    const int n = min((int64_t)nrow[s], tc);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const int4 dd = desc[(int64_t)s * tc + j];
      if (dd.x < 0 || dd.x >= tc) {
        atomicOr(meta2 + 1, 1);
        continue;
      }
      for (int r = 0; r < K; ++r) {
        const uint32_t word = (uint32_t)(r < 4 ? dd.y : dd.z);
        const int le = (int)((word >> (8 * (r & 3))) & 0xFFu);
        if (le == 0xFF) continue;
        if (le >= e_per) {
          atomicOr(meta2 + 1, 1);
          continue;
        }
        const int q = atomicAdd(&fill[s * e_per + le], 1);
        if (q >= cnt_s[s * e_per + le]) {  // more entries than the counts announced
          atomicOr(meta2 + 1, 1);
          continue;
        }
        const int pos = dst_off[s * e_per + le] + q;
        perm2[pos] = (int32_t)((int64_t)s * tc + j);
        ret2[pos] = ((int64_t)s << 32) | (int64_t)((int64_t)dd.x * K + r);
      }
    }
  }
}

// Return: each position's output row y[pos] stored into its source rank's
// slot (copy != 0), then the last CTA releases this rank's return flag on
// every rank.  With copy == 0 (the down GEMM stored the rows itself) one CTA
// only signals.
__global__ void __launch_bounds__(kDispatchThreads)
    ep_return_kernel(const float* __restrict__ y, const int64_t* __restrict__ ret2,
                     const int32_t* __restrict__ offsets2, int E, int H, int K, int64_t tc,
                     EpPeers p, int me, int N, int epoch, unsigned* __restrict__ ticket,
                     int32_t* __restrict__ err, int copy) {
  __shared__ bool last;
  const int64_t pos = blockIdx.x;
  if (copy && pos < offsets2[E]) {
    const int64_t dst = ret2[pos];
    const int s = (int)(dst >> 32);
    const int64_t sl = dst & 0xffffffffll;
    if (dst < 0 || s >= N || sl >= tc * K) {
      if (threadIdx.x == 0) atomicOr(err, 1);
    } else {
      const float4* src = reinterpret_cast<const float4*>(y + pos * H);
      float4* out = reinterpret_cast<float4*>(p.y_back[s] + sl * H);
      for (int c = threadIdx.x; c < H / 4; c += blockDim.x) out[c] = src[c];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  if (threadIdx.x < N) st_release_sys(p.flags[threadIdx.x] + N + me, epoch);
  if (threadIdx.x == 0) *ticket = 0;
}

// Small device <-> host transfers that must not queue behind bulk copies on
// the copy engines: a kernel stores into mapped pinned host memory, or
// writes a value passed as its argument.
__global__ void ep_to_host_kernel(const int32_t* __restrict__ src, int n,
                                  volatile int32_t* __restrict__ host) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) host[i] = src[i];
  __threadfence_system();
}

__global__ void ep_set_i64_kernel(int64_t* __restrict__ dst, int64_t v) { *dst = v; }

__global__ void ep_i64_to_host_kernel(const int64_t* __restrict__ src,
                                      volatile int64_t* __restrict__ host) {
  *host = *src;
  __threadfence_system();
}

// Bounded wait for every rank's return flag of this epoch.
__global__ void ep_wait_kernel(const int* __restrict__ flags, int N, int epoch,
                               uint64_t timeout_ns, int32_t* __restrict__ err) {
  if ((int)threadIdx.x < N && !wait_epoch(flags + N + threadIdx.x, epoch, timeout_ns))
    atomicOr(err, 2);
}

}  // namespace

// ---- host side ------------------------------------------------------------

int nccl_unique_id(uint8_t out[128]) {
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId id;
  const ncclResult_t r = g_nccl.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, 128);
  return GB_OK;
}

namespace {

size_t round256(size_t v) { return (v + 255) / 256 * 256; }

// All-gather of `bytes` bytes per rank through NCCL (host buffers in and out).
int allgather_host(Ep* ep, const void* mine, void* all, size_t bytes, cudaStream_t st,
                   const char* what) {
  uint8_t* dev = nullptr;
  GB_CU(cudaMalloc(&dev, bytes * (ep->size + 1)), what);
  int rc = GB_OK;
  cudaError_t ce = cudaMemcpyAsync(dev, mine, bytes, cudaMemcpyHostToDevice, st);
  if (ce == cudaSuccess) {
    rc = nccl_settle(ep, g_nccl.AllGather(dev, dev + bytes, bytes, ncclUint8, ep->comm, st), what);
    if (!rc) rc = stream_settle(ep, st, what);
    if (!rc) {
      ce = cudaMemcpy(all, dev + bytes, bytes * ep->size, cudaMemcpyDeviceToHost);
    }
  }
  cudaFree(dev);
  if (!rc && ce != cudaSuccess) rc = set_error(GB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(ce));
  return rc;
}

}  // namespace

int ep_init(Moe& m, const uint8_t* id_bytes) {
  int rc = load_nccl();
  if (rc) return rc;
  if (!id_bytes) return set_error(GB_ERR_INVALID_ARG, "ep_size > 1 needs nccl_id");
  if (m.ep_size > kMaxRanks)
    return set_error(GB_ERR_UNSUPPORTED, "ep_size %d > %d (one NVSwitch node)", m.ep_size,
                     kMaxRanks);
  const gb_moe_desc& d = m.desc;
  Ep* ep = new Ep();
  m.ep = ep;
  ep->rank = m.ep_rank;
  ep->size = m.ep_size;
  ep->e_per = d.n_experts / m.ep_size;
  if (d.ep_timeout_ms > 0) ep->timeout_ms = d.ep_timeout_ms;
  ncclUniqueId id;
  memcpy(&id, id_bytes, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  if ((rc = nccl_settle(ep, g_nccl.CommInitRankConfig(&ep->comm, ep->size, id, ep->rank, &cfg),
                        "ncclCommInitRankConfig")))
    return rc;
  cudaStream_t st = nullptr;
  GB_CU(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "EP setup stream");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } guard{st};

  // receive rows per source: the largest max_tokens of the ranks
  const int32_t mine = std::max(1, d.max_tokens);
  std::vector<int32_t> all(ep->size);
  if ((rc = allgather_host(ep, &mine, all.data(), sizeof mine, st, "agree on max_tokens")))
    return rc;
  ep->tc = *std::max_element(all.begin(), all.end());

  // the shared allocation and its CUDA IPC handle
  const int N = ep->size, E = d.n_experts, K = d.top_k;
  const int64_t H = d.hidden, tc = ep->tc;
  const size_t off_desc = round256((size_t)N * tc * H * sizeof(float));
  const size_t off_rows = off_desc + round256((size_t)N * tc * sizeof(int4));
  const size_t off_flags = off_rows + round256((size_t)N * sizeof(int));
  const size_t off_y = off_flags + round256((size_t)2 * N * sizeof(int));
  ep->sym_bytes = off_y + round256((size_t)tc * K * H * sizeof(float));
  if (cudaMalloc(&ep->sym, ep->sym_bytes) != cudaSuccess) {
    cudaGetLastError();
    ep->sym = nullptr;
    return set_error(GB_ERR_NO_MEMORY, "EP receive buffers (%zu bytes)", ep->sym_bytes);
  }
  GB_CU(cudaMemset(ep->sym, 0, ep->sym_bytes), "clear EP buffers");
  cudaIpcMemHandle_t h;
  GB_CU(cudaIpcGetMemHandle(&h, ep->sym), "cudaIpcGetMemHandle");
  std::vector<cudaIpcMemHandle_t> handles(N);
  if ((rc = allgather_host(ep, &h, handles.data(), sizeof h, st, "exchange EP buffer handles")))
    return rc;
  for (int p = 0; p < N; ++p) {
    char* base = static_cast<char*>(ep->sym);
    if (p != ep->rank) {
      GB_CU(cudaIpcOpenMemHandle(&ep->peer_base[p], handles[p], cudaIpcMemLazyEnablePeerAccess),
            "cudaIpcOpenMemHandle");
      base = static_cast<char*>(ep->peer_base[p]);
    }
    ep->peers.recv_x[p] = reinterpret_cast<float*>(base);
    ep->peers.desc[p] = reinterpret_cast<int4*>(base + off_desc);
    ep->peers.rows[p] = reinterpret_cast<int*>(base + off_rows);
    ep->peers.flags[p] = reinterpret_cast<int*>(base + off_flags);
    ep->peers.y_back[p] = reinterpret_cast<float*>(base + off_y);
  }

  GB_CU(cudaMalloc(&ep->cnt_recv, sizeof(int32_t) * E), "EP counts");
  GB_CU(cudaMalloc(&ep->counts2, sizeof(int32_t) * E), "EP counts");
  GB_CU(cudaMalloc(&ep->offsets2, sizeof(int32_t) * (E + 1)), "EP offsets");
  GB_CU(cudaMalloc(&ep->active2, sizeof(int32_t) * E), "EP active");
  GB_CU(cudaMalloc(&ep->meta2, sizeof(int32_t) * 4), "EP meta");
  GB_CU(cudaMemset(ep->meta2, 0, sizeof(int32_t) * 4), "EP meta");
  GB_CU(cudaMemset(ep->offsets2, 0, sizeof(int32_t) * (E + 1)), "EP offsets");
  GB_CU(cudaMalloc(&ep->slot, sizeof(int32_t) * (size_t)tc * N), "EP slots");
  GB_CU(cudaMalloc(&ep->nrows, sizeof(int32_t) * std::max(N, 2)), "EP row counts");
  GB_CU(cudaMalloc(&ep->tickets, sizeof(unsigned) * 2), "EP tickets");
  GB_CU(cudaMemset(ep->tickets, 0, sizeof(unsigned) * 2), "EP tickets");
  GB_CU(cudaHostAlloc(&ep->host, sizeof(int32_t) * std::max(E, 2), cudaHostAllocMapped),
        "EP mapped counts");
  GB_CU(cudaHostGetDevicePointer(&ep->host_dev, ep->host, 0), "EP mapped counts");
  GB_CU(cudaDeviceSynchronize(), "EP setup");
  return GB_OK;
}

int32_t* ep_meta(Moe& m) { return m.ep ? m.ep->meta2 : nullptr; }

int* ep_arrivals(Moe& m) { return m.ep ? m.ep->eb.mx_arrivals : nullptr; }

int ep_agree_max(Moe& m, int64_t v, int64_t* out, cudaStream_t st) {
  Ep* ep = m.ep;
  if (ep->broken)
    return set_error(GB_ERR_NCCL, "the expert-parallel communicator was aborted by an earlier "
                                  "failure; destroy and recreate the handle on every rank");
  int64_t* dev = reinterpret_cast<int64_t*>(ep->nrows);  // free between forwards
  ep_set_i64_kernel<<<1, 1, 0, st>>>(dev, v);
  GB_CU(cudaGetLastError(), "agree on T");
  int rc = nccl_settle(ep, g_nccl.AllReduce(dev, dev, 1, ncclInt64, ncclMax, ep->comm, st),
                       "agree on T");
  if (rc) return rc;
  ep_i64_to_host_kernel<<<1, 1, 0, st>>>(dev, reinterpret_cast<int64_t*>(ep->host_dev));
  GB_CU(cudaGetLastError(), "agree on T");
  if ((rc = stream_settle(ep, st, "agree on T"))) return rc;
  *out = *reinterpret_cast<volatile int64_t*>(ep->host);
  return GB_OK;
}

int64_t ep_capacity(const Moe& m) { return m.ep ? m.ep->tc : 0; }

void ep_destroy(Moe& m) {
  Ep* ep = m.ep;
  if (!ep) return;
  cudaDeviceSynchronize();
  if (ep->comm) {
    // finalize (non-blocking: poll it within the deadline), then free; a
    // finalize that does not finish is aborted instead
    ncclResult_t st = g_nccl.CommFinalize(ep->comm);
    const auto deadline = Clock::now() + std::chrono::milliseconds(ep->timeout_ms);
    while (st == ncclInProgress && Clock::now() < deadline) {
      std::this_thread::sleep_for(std::chrono::microseconds(100));
      if (g_nccl.CommGetAsyncError(ep->comm, &st) != ncclSuccess) st = ncclSystemError;
    }
    if (st == ncclSuccess)
      g_nccl.CommDestroy(ep->comm);
    else
      g_nccl.CommAbort(ep->comm);
    ep->comm = nullptr;
  }
  for (void*& b : ep->peer_base)
    if (b) cudaIpcCloseMemHandle(b);
  cudaFree(ep->sym);
  cudaFree(ep->cnt_recv);
  cudaFree(ep->counts2);
  cudaFree(ep->offsets2);
  cudaFree(ep->active2);
  cudaFree(ep->meta2);
  cudaFree(ep->slot);
  cudaFree(ep->nrows);
  cudaFree(ep->tickets);
  cudaFreeHost(ep->host);
  cudaFree(ep->perm2);
  cudaFree(ep->ret2);
  free_expert_bufs(ep->eb);
  delete ep;
  m.ep = nullptr;
}

static int ensure_positions(Moe& m, int64_t R, cudaStream_t st) {
  Ep* ep = m.ep;
  if (R <= ep->r_cap) return GB_OK;
  GB_CU(cudaStreamSynchronize(st), "synchronise before EP buffer growth");
  const int64_t cap = std::max<int64_t>(R, 2 * ep->r_cap);
  cudaFree(ep->perm2);
  cudaFree(ep->ret2);
  ep->perm2 = nullptr;
  ep->ret2 = nullptr;
  ep->r_cap = 0;
  if (cudaMalloc(&ep->perm2, sizeof(int32_t) * (size_t)cap) != cudaSuccess ||
      cudaMalloc(&ep->ret2, sizeof(int64_t) * (size_t)cap) != cudaSuccess) {
    cudaGetLastError();
    return set_error(GB_ERR_NO_MEMORY, "EP position buffers for %lld positions", (long long)cap);
  }
  int rc = alloc_expert_bufs(m, ep->eb, cap);
  if (rc) return rc;
  ep->r_cap = cap;
  return GB_OK;
}

int ep_forward(Moe& m, const float* x, int64_t T, float* out, cudaStream_t st) {
  Ep* ep = m.ep;
  const gb_moe_desc& d = m.desc;
  const int E = d.n_experts, K = d.top_k, H = d.hidden, N = ep->size, e_per = ep->e_per;
  Workspace& ws = m.ws;
  if (ep->broken)
    return set_error(GB_ERR_NCCL,
                     "the expert-parallel communicator was aborted by an earlier failure; "
                     "destroy and recreate the handle on every rank");
  if (T > ep->tc)
    return set_error(GB_ERR_INVALID_ARG,
                     "T = %lld exceeds the expert-parallel capacity of %lld tokens per rank "
                     "(the largest max_tokens given at create)",
                     (long long)T, (long long)ep->tc);
  const int epoch = ++ep->epoch;
  const uint64_t timeout_ns = (uint64_t)ep->timeout_ms * 1000000ull;
  int rc;

  // 1. count exchange: positions per local expert from every source
  if ((rc = nccl_settle(ep, g_nccl.GroupStart(), "ncclGroupStart"))) return rc;
  for (int p = 0; p < N; ++p) {
    ncclResult_t r = g_nccl.Send(ws.counts + p * e_per, (size_t)e_per, ncclInt32, p, ep->comm, st);
    if (r == ncclSuccess || r == ncclInProgress)
      r = g_nccl.Recv(ep->cnt_recv + p * e_per, (size_t)e_per, ncclInt32, p, ep->comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
      g_nccl.GroupEnd();
      abort_comm(ep);
      return nccl_err(r, "count exchange");
    }
  }
  if ((rc = nccl_settle(ep, g_nccl.GroupEnd(), "count exchange"))) return rc;
  ep_to_host_kernel<<<1, 256, 0, st>>>(ep->cnt_recv, E, ep->host_dev);
  GB_CU(cudaGetLastError(), "read received counts");
  if ((rc = stream_settle(ep, st, "count exchange"))) return rc;
  int64_t R = 0;
  for (int i = 0; i < N * e_per; ++i) R += reinterpret_cast<volatile int32_t*>(ep->host)[i];
  if ((rc = ensure_positions(m, std::max<int64_t>(R, 1), st))) return rc;

  // 2. dispatch: each token's row once per destination rank, by peer stores
  if (T > 0) {
    ep_slots_kernel<<<N, 1024, 0, st>>>(ws.idx, (int)T, K, e_per, N, ep->slot, ep->nrows);
  } else {
    GB_CU(cudaMemsetAsync(ep->nrows, 0, sizeof(int32_t) * N, st), "clear EP row counts");
  }
  ep_dispatch_kernel<<<(unsigned)std::max<int64_t>(T, 1), kDispatchThreads, 0, st>>>(
      x, (int)T, H, K, e_per, ws.idx, ep->slot, ep->nrows, ep->rank, N, ep->tc, ep->peers, epoch,
      ep->tickets);
  GB_CU(cudaGetLastError(), "EP dispatch launch");

  // 3. grouping of the received rows
  {
    const size_t smem = sizeof(int) * 3 * (size_t)N * e_per;
    ep_plan_kernel<<<1, 1024, smem, st>>>(ep->peers.flags[ep->rank], epoch, timeout_ns,
                                          ep->peers.rows[ep->rank], ep->peers.desc[ep->rank],
                                          ep->tc, ep->cnt_recv, N, e_per, m.e_begin, E, K,
                                          ep->r_cap, ep->counts2, ep->offsets2, ep->active2,
                                          ep->meta2, ep->perm2, ep->ret2);
    GB_CU(cudaGetLastError(), "EP plan launch");
  }

  // 4. experts on the received rows
  Groups g;
  g.counts = ep->counts2;
  g.offsets = ep->offsets2;
  g.active = ep->active2;
  g.meta = ep->meta2;
  g.perm = ep->perm2;
  g.perm_div = 1;
  g.rows = R;
  g.max_active = (int)std::min<int64_t>(e_per, R);
  g.max_per_expert = R;
  g.out_rows = nullptr;
  g.ret_dst = ep->ret2;
  for (int p = 0; p < N; ++p) g.ret_base[p] = ep->peers.y_back[p];
  g.ret_slots = ep->tc * K;
  bool stored = false;
  if (R > 0 && (rc = run_experts(m, g, ep->peers.recv_x[ep->rank], T, ep->eb, st, &stored)))
    return rc;
  if ((rc = mark_stage(m, 4, st))) return rc;

  // 5. return (rows the down kernel did not store itself) and its flags
  const bool copy = R > 0 && !stored;
  ep_return_kernel<<<(unsigned)(copy ? R : 1), kDispatchThreads, 0, st>>>(
      ep->eb.y, ep->ret2, ep->offsets2, E, H, K, ep->tc, ep->peers, ep->rank, N, epoch,
      ep->tickets + 1, ep->meta2 + 1, copy ? 1 : 0);
  GB_CU(cudaGetLastError(), "EP return launch");

  // 6. every rank's rows are back: combine in the single-GPU order
  ep_wait_kernel<<<1, 32, 0, st>>>(ep->peers.flags[ep->rank], N, epoch, timeout_ns, ep->meta2 + 1);
  GB_CU(cudaGetLastError(), "EP wait launch");
  if (T > 0)
    GB_CU(launch_combine(m, T, ws, ep->peers.y_back[ep->rank], out, st, /*slots=*/true),
          "combine launch");
  m.launches += 6;
  return GB_OK;
}

}  // namespace gb
