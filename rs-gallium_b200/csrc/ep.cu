// ep.cu -- expert parallelism across the GPUs of one node (one process per GPU).
//
// No counterpart in the reference, which runs on one device.  Rank r owns
// experts [r*E/N, (r+1)*E/N) and routes its own tokens.  Because the local
// grouping is expert-ascending, the rows bound for rank d are one contiguous
// range [offsets[d*E/N], offsets[(d+1)*E/N]) of the grouped order, so:
//
//   1. count exchange   per-expert counts, E/N ints to every peer (NCCL)
//   2. sizes            one device->host copy of the counts; host sums them
//   3. dispatch         grouped ncclSend/ncclRecv of f32 activation rows
//   4. local grouping   a kernel orders the received rows by local expert
//                       (expert ascending, then source rank, then the
//                       source's order) without moving them (an index list)
//   5. experts          the same expert kernels as one GPU, writing each
//                       output row back at its received slot
//   6. return           the reverse grouped ncclSend/ncclRecv
//   7. combine          the single-GPU combine, rank order fixed per token
//
// NCCL is opened at run time (dlopen of libnccl.so.2, the copy PyTorch has
// already loaded when there is one), so single-GPU use needs no NCCL.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "moe_internal.h"

namespace gb {

namespace {

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
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
  GB_SYM(CommInitRank, "ncclCommInitRank")
  GB_SYM(CommDestroy, "ncclCommDestroy")
  GB_SYM(CommAbort, "ncclCommAbort")
  GB_SYM(GroupStart, "ncclGroupStart")
  GB_SYM(GroupEnd, "ncclGroupEnd")
  GB_SYM(Send, "ncclSend")
  GB_SYM(Recv, "ncclRecv")
  GB_SYM(GetErrorString, "ncclGetErrorString")
#undef GB_SYM
  g_nccl = a;
  return GB_OK;
}

int nccl_err(ncclResult_t r, const char* what) {
  return set_error(GB_ERR_NCCL, "%s: %s", what,
                   g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error");
}

#define GB_NCCL(call, what)                          \
  do {                                               \
    ncclResult_t _r = (call);                        \
    if (_r != ncclSuccess) return nccl_err(_r, what); \
  } while (0)

#define GB_CU(call, what)                                                                   \
  do {                                                                                      \
    cudaError_t _e = (call);                                                                \
    if (_e != cudaSuccess)                                                                  \
      return set_error(GB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e));               \
  } while (0)

// send_x[p] = x[perm[p] / k]: activation rows in grouped (destination) order.
__global__ void gather_rows_kernel(const float* __restrict__ x, const int32_t* __restrict__ perm,
                                   int top_k, int H, float* __restrict__ out) {
  const int64_t p = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(x + (int64_t)(perm[p] / top_k) * H);
  float4* dst = reinterpret_cast<float4*>(out + p * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
}

// Received rows -> grouped view.  cnt[s][e] rows of local expert e came from
// source s, stored source-major, expert-ascending inside each source.
// counts2/offsets2 are indexed by global expert id; perm2[pos] is the
// received row at grouped position pos.
__global__ void ep_plan_kernel(const int32_t* __restrict__ cnt, int n_src, int e_per, int e_begin,
                               int E, int32_t* __restrict__ counts2, int32_t* __restrict__ offsets2,
                               int32_t* __restrict__ active2, int32_t* __restrict__ meta2,
                               int32_t* __restrict__ perm2) {
  extern __shared__ int32_t sh[];
  int32_t* c = sh;                       // [n_src][e_per]
  int32_t* src_off = c + n_src * e_per;  // [n_src][e_per] first received row of (s, e)
  int32_t* dst_off = src_off + n_src * e_per;  // [n_src][e_per] first grouped position of (s, e)
  for (int i = threadIdx.x; i < n_src * e_per; i += blockDim.x) c[i] = cnt[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int s = 0; s < n_src; ++s)
      for (int e = 0; e < e_per; ++e) {
        src_off[s * e_per + e] = run;
        run += c[s * e_per + e];
      }
    int pos = 0, nact = 0;
    for (int g = 0; g < E; ++g) {
      offsets2[g] = pos;
      const int e = g - e_begin;
      int n = 0;
      if (e >= 0 && e < e_per) {
        for (int s = 0; s < n_src; ++s) {
          dst_off[s * e_per + e] = pos + n;
          n += c[s * e_per + e];
        }
        if (n > 0) active2[nact++] = g;
      }
      counts2[g] = n;
      pos += n;
    }
    offsets2[E] = pos;
    meta2[0] = nact;
    meta2[1] = 0;
  }
  __syncthreads();
  // one warp per (source, expert) segment
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int seg = warp; seg < n_src * e_per; seg += nw) {
    const int n = c[seg], so = src_off[seg], d = dst_off[seg];
    for (int i = lane; i < n; i += 32) perm2[d + i] = so + i;
  }
}

}  // namespace

struct Ep {
  ncclComm_t comm = nullptr;
  int rank = 0, size = 1, e_per = 0;
  int32_t* cnt_recv = nullptr;  // [size][e_per]
  int32_t* counts2 = nullptr;   // [E]
  int32_t* offsets2 = nullptr;  // [E+1]
  int32_t* active2 = nullptr;   // [E]
  int32_t* meta2 = nullptr;     // [4]
  int32_t* host = nullptr;      // pinned: [E] local counts, [E] received counts
  int32_t* perm2 = nullptr;     // [r_cap]
  float* recv_x = nullptr;      // [r_cap][H]
  int64_t r_cap = 0;
  ExpertBufs eb;                // r_cap positions; y in received-row order
};

int nccl_unique_id(uint8_t out[128]) {
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId id;
  GB_NCCL(g_nccl.GetUniqueId(&id), "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, 128);
  return GB_OK;
}

int ep_init(Moe& m, const uint8_t* id_bytes) {
  int rc = load_nccl();
  if (rc) return rc;
  if (!id_bytes) return set_error(GB_ERR_INVALID_ARG, "ep_size > 1 needs nccl_id");
  Ep* ep = new Ep();
  ep->rank = m.ep_rank;
  ep->size = m.ep_size;
  ep->e_per = m.desc.n_experts / m.ep_size;
  m.ep = ep;
  ncclUniqueId id;
  memcpy(&id, id_bytes, 128);
  GB_NCCL(g_nccl.CommInitRank(&ep->comm, ep->size, id, ep->rank), "ncclCommInitRank");
  const int E = m.desc.n_experts;
  GB_CU(cudaMalloc(&ep->cnt_recv, sizeof(int32_t) * E), "EP counts");
  GB_CU(cudaMalloc(&ep->counts2, sizeof(int32_t) * E), "EP counts");
  GB_CU(cudaMalloc(&ep->offsets2, sizeof(int32_t) * (E + 1)), "EP offsets");
  GB_CU(cudaMalloc(&ep->active2, sizeof(int32_t) * E), "EP active");
  GB_CU(cudaMalloc(&ep->meta2, sizeof(int32_t) * 4), "EP meta");
  GB_CU(cudaMemset(ep->meta2, 0, sizeof(int32_t) * 4), "EP meta");
  GB_CU(cudaMallocHost(&ep->host, sizeof(int32_t) * 2 * E), "EP pinned counts");
  return GB_OK;
}

int32_t* ep_meta(Moe& m) { return m.ep ? m.ep->meta2 : nullptr; }

void ep_destroy(Moe& m) {
  Ep* ep = m.ep;
  if (!ep) return;
  if (ep->comm && g_nccl.CommDestroy) g_nccl.CommDestroy(ep->comm);
  cudaFree(ep->cnt_recv);
  cudaFree(ep->counts2);
  cudaFree(ep->offsets2);
  cudaFree(ep->active2);
  cudaFree(ep->meta2);
  cudaFreeHost(ep->host);
  cudaFree(ep->perm2);
  cudaFree(ep->recv_x);
  free_expert_bufs(ep->eb);
  delete ep;
  m.ep = nullptr;
}

static int ensure_recv(Moe& m, int64_t R, cudaStream_t st) {
  Ep* ep = m.ep;
  if (R <= ep->r_cap) return GB_OK;
  GB_CU(cudaStreamSynchronize(st), "synchronise before EP buffer growth");
  const int64_t cap = std::max<int64_t>(R, 2 * ep->r_cap);
  cudaFree(ep->perm2);
  cudaFree(ep->recv_x);
  ep->perm2 = nullptr;
  ep->recv_x = nullptr;
  ep->r_cap = 0;
  if (cudaMalloc(&ep->perm2, sizeof(int32_t) * (size_t)cap) != cudaSuccess ||
      cudaMalloc(&ep->recv_x, sizeof(float) * (size_t)cap * m.desc.hidden) != cudaSuccess) {
    cudaGetLastError();
    return set_error(GB_ERR_NO_MEMORY, "EP receive buffers for %lld rows", (long long)cap);
  }
  int rc = alloc_expert_bufs(m, ep->eb, cap);
  if (rc) return rc;
  ep->r_cap = cap;
  return GB_OK;
}

int ep_forward(Moe& m, const float* x, int64_t T, float* out, cudaStream_t st) {
  Ep* ep = m.ep;
  const gb_moe_desc& d = m.desc;
  const int E = d.n_experts, K = d.top_k, H = d.hidden, N = ep->size, ep_ = ep->e_per;
  Workspace& ws = m.ws;
  const int64_t rows_out = T * K;

  // 1. activation rows in grouped order, and the count exchange
  if (rows_out > 0) {
    gather_rows_kernel<<<(unsigned)rows_out, 256, 0, st>>>(x, ws.perm, K, H, ws.send_x);
    GB_CU(cudaGetLastError(), "EP gather launch");
  }
  GB_NCCL(g_nccl.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < N; ++p) {
    GB_NCCL(g_nccl.Send(ws.counts + p * ep_, (size_t)ep_, ncclInt32, p, ep->comm, st), "ncclSend counts");
    GB_NCCL(g_nccl.Recv(ep->cnt_recv + p * ep_, (size_t)ep_, ncclInt32, p, ep->comm, st), "ncclRecv counts");
  }
  GB_NCCL(g_nccl.GroupEnd(), "ncclGroupEnd counts");

  // 2. sizes on the host
  GB_CU(cudaMemcpyAsync(ep->host, ws.counts, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, st),
        "copy counts");
  GB_CU(cudaMemcpyAsync(ep->host + E, ep->cnt_recv, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, st),
        "copy received counts");
  GB_CU(cudaStreamSynchronize(st), "synchronise counts");
  std::vector<int64_t> send_rows(N), send_off(N), recv_rows(N), recv_off(N);
  int64_t run = 0;
  for (int p = 0; p < N; ++p) {
    int64_t sr = 0, rr = 0;
    for (int e = 0; e < ep_; ++e) {
      sr += ep->host[p * ep_ + e];
      rr += ep->host[E + p * ep_ + e];
    }
    send_rows[p] = sr;
    recv_rows[p] = rr;
    recv_off[p] = run;
    run += rr;
  }
  int64_t so = 0;
  for (int p = 0; p < N; ++p) {
    send_off[p] = so;
    so += send_rows[p];
  }
  const int64_t R = run;
  int rc = ensure_recv(m, std::max<int64_t>(R, 1), st);
  if (rc) return rc;

  // 3. dispatch
  GB_NCCL(g_nccl.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < N; ++p) {
    if (send_rows[p])
      GB_NCCL(g_nccl.Send(ws.send_x + send_off[p] * H, (size_t)(send_rows[p] * H), ncclFloat32, p,
                          ep->comm, st),
              "ncclSend rows");
    if (recv_rows[p])
      GB_NCCL(g_nccl.Recv(ep->recv_x + recv_off[p] * H, (size_t)(recv_rows[p] * H), ncclFloat32, p,
                          ep->comm, st),
              "ncclRecv rows");
  }
  GB_NCCL(g_nccl.GroupEnd(), "ncclGroupEnd rows");

  // 4. local grouping of the received rows
  {
    const size_t smem = sizeof(int32_t) * 3 * (size_t)N * ep_;
    ep_plan_kernel<<<1, 256, smem, st>>>(ep->cnt_recv, N, ep_, m.e_begin, E, ep->counts2,
                                         ep->offsets2, ep->active2, ep->meta2, ep->perm2);
    GB_CU(cudaGetLastError(), "EP plan launch");
  }

  // 5. experts; outputs land at their received slots
  Groups g;
  g.counts = ep->counts2;
  g.offsets = ep->offsets2;
  g.active = ep->active2;
  g.meta = ep->meta2;
  g.perm = ep->perm2;
  g.perm_div = 1;
  g.rows = R;
  g.max_active = (int)std::min<int64_t>(ep_, R);
  g.max_per_expert = R;
  g.out_rows = ep->perm2;
  if (R > 0 && (rc = run_experts(m, g, ep->recv_x, T, ep->eb, st))) return rc;
  if ((rc = mark_stage(m, 4, st))) return rc;

  // 6. return the rows to their sources
  GB_NCCL(g_nccl.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < N; ++p) {
    if (recv_rows[p])
      GB_NCCL(g_nccl.Send(ep->eb.y + recv_off[p] * H, (size_t)(recv_rows[p] * H), ncclFloat32, p,
                          ep->comm, st),
              "ncclSend results");
    if (send_rows[p])
      GB_NCCL(g_nccl.Recv(ws.y_back + send_off[p] * H, (size_t)(send_rows[p] * H), ncclFloat32, p,
                          ep->comm, st),
              "ncclRecv results");
  }
  GB_NCCL(g_nccl.GroupEnd(), "ncclGroupEnd results");

  // 7. combine
  if (T > 0) GB_CU(launch_combine(m, T, ws, ws.y_back, out, st), "combine launch");
  m.launches += 3;
  return GB_OK;
}

}  // namespace gb
