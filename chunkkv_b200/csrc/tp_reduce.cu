// Tensor-parallel exchange over NVLink peer memory, without a collective library:
// every rank's row-parallel GEMM (ckv_linear_partial) writes its partial rows into its
// own buffer and signals; this kernel, on the rank that owns a 128-row block (block b ->
// rank b % ranks), reads the ranks' partial rows of that block over NVLink, sums them in
// a fixed rank order, adds them to the residual stream, and writes the finished h rows
// to every rank (an all-gather by NVLink stores).  Together they replace the NCCL all-reduce after o_proj and down_proj
// (torch_engine.py:70-76 residual adds), with the same h on every rank; the next
// RMSNorm then runs locally on every rank (ckv_rmsnorm), which costs less than sending
// the normed rows too.
//
// Ordering: the GEMM's last CTA adds 1 to each rank's partial counter for its own rank
// (release, system scope) after every CTA has fenced its stores; this kernel's CTAs wait
// (acquire, bounded) for all ranks' counters to reach `epoch`.  Its own last CTA then
// signals every rank's gather counter the same way and waits until all ranks' gather
// counters reached `epoch`, so when the kernel ends every rank's h and x rows are here.
// Every wait is bounded (2 s); a wait that runs out sets CKV_DEV_ERR_WAIT_TIMEOUT and the
// kernel goes on without the data (the host raises on the error word).
//
// Also here: CUDA IPC helpers that map one allocation of each rank into the others'
// address spaces (plain peer mappings, no multicast objects).
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(tp_reduce)

namespace ckv {
namespace {

constexpr int kRowBlock = 128;

struct ReduceArgs {
  const uint64_t* part;   // [ranks] partial rows of each rank, [M][hidden] bf16
  int rank, ranks;
  int M, hidden;
  const uint16_t* h;      // this rank's residual stream [M][hidden]
  const uint64_t* h_peer; // [ranks] h of each rank (this rank's own at index rank)
  const unsigned* recv_cnt;    // this rank's receive counters [ranks]
  unsigned* gather_cnt;        // this rank's gather counters [ranks]
  const uint64_t* gather_peer; // [ranks] address of each rank's gather counters
  unsigned* ticket;            // this rank's CTA ticket (left at 0)
  unsigned epoch;              // counters' value once this exchange is complete
};

// One warp per (owned row, segment of kSegVecs 16-byte vectors), persistent CTAs of kWarps
// warps, so the remote reads of a row spread over several warps.  Owned row i: block
// rank + (i / 128) * ranks, row i % 128 in it.
constexpr int kWarps = 8;
constexpr int kSegVecs = 128;
// T ranks (compile time), U vectors per lane in flight per rank
template <int T, int U>
__global__ void __launch_bounds__(kWarps * 32) reduce_gather_kernel(ReduceArgs a, int n_owned) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int q = 0; q < a.ranks && ok; ++q) ok = wait_counter(a.recv_cnt + q, a.epoch, &g_err_word);
    if (!ok) atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int vecs = a.hidden / 8;  // 16-byte vectors per row
  const int segs = (vecs + kSegVecs - 1) / kSegVecs;
  const int items = n_owned * segs;
  if (s_ok) {
    for (int it = blockIdx.x * kWarps + (threadIdx.x >> 5); it < items; it += gridDim.x * kWarps) {
      const int i = it / segs, sg = it - (it / segs) * segs;
      const int row = (a.rank + (i / kRowBlock) * a.ranks) * kRowBlock + (i % kRowBlock);
      if (row >= a.M) continue;
      const int64_t rbase = int64_t(row) * a.hidden;
      const int c_end = min(vecs, (sg + 1) * kSegVecs);
      for (int c0 = sg * kSegVecs; c0 < c_end; c0 += 32 * U) {
        // all ranks' partials of U vectors per lane in flight before any add
        uint4 d[T][U];
#pragma unroll
        for (int q = 0; q < T; ++q)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int c = c0 + lane + 32 * u;
            d[q][u] = c < c_end ? __ldcg(reinterpret_cast<const uint4*>(a.part[q] + rbase * 2) + c)
                                : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + lane + 32 * u;
          if (c >= c_end) continue;
          // fixed rank order, fp32: the same bits on every rank; then h = bf16(h + bf16(sum))
          // into every rank's copy of the row, this rank's included
          float acc[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
          for (int q = 0; q < T; ++q) {
            const uint32_t* pw = reinterpret_cast<const uint32_t*>(&d[q][u]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[2 * e] = __fadd_rn(acc[2 * e], lo_bf(pw[e]));
              acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], hi_bf(pw[e]));
            }
          }
          const uint4 old = reinterpret_cast<const uint4*>(a.h + rbase)[c];
          const uint32_t* po = reinterpret_cast<const uint32_t*>(&old);
          uint4 hv;
          uint32_t* pn = reinterpret_cast<uint32_t*>(&hv);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pn[e] = pack_bf2(__fadd_rn(lo_bf(po[e]), bf16_round(acc[2 * e])),
                             __fadd_rn(hi_bf(po[e]), bf16_round(acc[2 * e + 1])));
#pragma unroll
          for (int q = 0; q < T; ++q) reinterpret_cast<uint4*>(a.h_peer[q] + rbase * 2)[c] = hv;
        }
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(a.ticket, 1u);
    if (t == gridDim.x - 1) {
      // every CTA of this rank has written its rows: tell all ranks, then wait for theirs
      __threadfence_system();
      for (int q = 0; q < a.ranks; ++q)
        red_release_sys_add(reinterpret_cast<unsigned*>(a.gather_peer[q]) + a.rank, 1u);
      *a.ticket = 0u;
      bool ok = true;
      for (int q = 0; q < a.ranks && ok; ++q) ok = wait_counter(a.gather_cnt + q, a.epoch, &g_err_word);
      if (!ok) atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
    }
  }
}

// rows of [0, M) in row blocks owned by `rank`
int owned_rows(int M, int rank, int ranks) {
  const int blocks = ceil_div(M, kRowBlock);
  int n = 0;
  for (int b = rank; b < blocks; b += ranks) n += std::min(kRowBlock, M - b * kRowBlock);
  return n;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  CKV_REQUIRE(bytes > 0 && ptr && handle, "ckv_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, size_t(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, size_t(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_error("ckv_ipc_alloc(%lld): %s", (long long)bytes, cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return CKV_OK;
}

int ckv_ipc_open(const void* handle, void** ptr) {
  CKV_REQUIRE(handle && ptr, "ckv_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("ckv_ipc_open: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

int ckv_ipc_close(void* ptr) {
  CKV_REQUIRE(ptr, "ckv_ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("ckv_ipc_close: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

int ckv_ipc_free(void* ptr) {
  CKV_REQUIRE(ptr, "ckv_ipc_free: null pointer");
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("ckv_ipc_free: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

int ckv_reduce_add_gather(const uint64_t* part_peer, int rank, int ranks, int m, int hidden,
                          const uint16_t* h, const uint64_t* h_peer, const uint32_t* part_cnt,
                          uint32_t* gather_cnt, const uint64_t* gather_peer, uint32_t* ticket,
                          uint32_t epoch, ckv_stream_t stream) {
  CKV_REQUIRE(part_peer && h && h_peer && part_cnt && gather_cnt && gather_peer && ticket,
              "ckv_reduce_add_gather: null pointer");
  CKV_REQUIRE(ranks >= 1 && ranks <= CKV_MAX_RANKS && rank >= 0 && rank < ranks,
              "ckv_reduce_add_gather: rank %d of %d", rank, ranks);
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0, "ckv_reduce_add_gather: hidden %d not a multiple of 8",
              hidden);
  CKV_REQUIRE(aligned16(h), "ckv_reduce_add_gather: h must be 16-byte aligned");
  if (m <= 0) return CKV_OK;
  ReduceArgs a{part_peer, rank, ranks, m, hidden, h, h_peer,
               reinterpret_cast<const unsigned*>(part_cnt), reinterpret_cast<unsigned*>(gather_cnt),
               gather_peer, reinterpret_cast<unsigned*>(ticket), epoch};
  // every rank launches at least one CTA, so every rank signals its gather counters
  const int n_owned = owned_rows(m, rank, ranks);
  const int items = n_owned * ceil_div(hidden / 8, kSegVecs);
  const int grid = std::max(1, std::min(ceil_div(items, kWarps), 8 * num_sms()));
  cudaStream_t s = as_stream(stream);
  switch (ranks) {
    case 1: reduce_gather_kernel<1, 4><<<grid, kWarps * 32, 0, s>>>(a, n_owned); break;
    case 2: reduce_gather_kernel<2, 4><<<grid, kWarps * 32, 0, s>>>(a, n_owned); break;
    case 4: reduce_gather_kernel<4, 2><<<grid, kWarps * 32, 0, s>>>(a, n_owned); break;
    case 8: reduce_gather_kernel<8, 1><<<grid, kWarps * 32, 0, s>>>(a, n_owned); break;
    default:
      set_error("ckv_reduce_add_gather: %d ranks (1, 2, 4 or 8)", ranks);
      return CKV_ERR_UNSUPPORTED;
  }
  CKV_LAUNCH_CHECK("ckv_reduce_add_gather");
  return CKV_OK;
}

}  // extern "C"
