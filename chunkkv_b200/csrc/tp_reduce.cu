// Tensor-parallel exchange over NVLink peer memory, without a collective library:
// the row-parallel GEMM (ckv_linear_push) stores each partial tile straight into the
// receive buffer of the rank that owns its 128-row block; this kernel, on the owning
// rank, sums the ranks' partial rows in a fixed rank order, adds them to the residual
// stream, and writes the finished h rows to every rank (an all-gather by NVLink
// stores).  Together they replace the NCCL all-reduce after o_proj and down_proj
// (torch_engine.py:70-76 residual adds), with the same h on every rank; the next
// RMSNorm then runs locally on every rank (ckv_rmsnorm), which costs less than sending
// the normed rows too.
//
// Ordering: the GEMM's last CTA adds 1 to each rank's receive counter for its own rank
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
  const uint16_t* recv;   // this rank's receive buffer: [ranks][slot] bf16
  int64_t slot;           // elements per source slot
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

// One warp per owned row, persistent CTAs of kWarps warps.  Owned row i: block
// rank + (i / 128) * ranks, row i % 128 in it.
constexpr int kWarps = 8;
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
  if (s_ok) {
    for (int i = blockIdx.x * kWarps + (threadIdx.x >> 5); i < n_owned; i += gridDim.x * kWarps) {
      const int row = (a.rank + (i / kRowBlock) * a.ranks) * kRowBlock + (i % kRowBlock);
      if (row >= a.M) continue;
      // fixed rank order, fp32: the same bits on every rank; then h = bf16(h + bf16(sum))
      // into every rank's copy of the row, this rank's included
      const int64_t rbase = int64_t(row) * a.hidden;
#pragma unroll 4
      for (int c = lane; c < vecs; c += 32) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        for (int q = 0; q < a.ranks; ++q) {
          const uint4 d = __ldcg(reinterpret_cast<const uint4*>(a.recv + q * a.slot + rbase) + c);
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(&d);
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
        for (int q = 0; q < a.ranks; ++q) reinterpret_cast<uint4*>(a.h_peer[q] + rbase * 2)[c] = hv;
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

int ckv_reduce_add_gather(const uint16_t* recv, int64_t slot_elems, int rank, int ranks, int m,
                          int hidden, const uint16_t* h, const uint64_t* h_peer,
                          const uint32_t* recv_cnt, uint32_t* gather_cnt, const uint64_t* gather_peer,
                          uint32_t* ticket, uint32_t epoch, ckv_stream_t stream) {
  CKV_REQUIRE(recv && h && h_peer && recv_cnt && gather_cnt && gather_peer && ticket,
              "ckv_reduce_add_gather: null pointer");
  CKV_REQUIRE(ranks >= 1 && ranks <= CKV_MAX_RANKS && rank >= 0 && rank < ranks,
              "ckv_reduce_add_gather: rank %d of %d", rank, ranks);
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0, "ckv_reduce_add_gather: hidden %d not a multiple of 8",
              hidden);
  CKV_REQUIRE(aligned16(recv) && aligned16(h) && slot_elems % 8 == 0 && slot_elems >= int64_t(m) * hidden,
              "ckv_reduce_add_gather: alignment or slot size");
  if (m <= 0) return CKV_OK;
  ReduceArgs a{recv, slot_elems, rank, ranks, m, hidden, h, h_peer,
               reinterpret_cast<const unsigned*>(recv_cnt), reinterpret_cast<unsigned*>(gather_cnt),
               gather_peer, reinterpret_cast<unsigned*>(ticket), epoch};
  // every rank launches at least one CTA, so every rank signals its gather counters
  const int n_owned = owned_rows(m, rank, ranks);
  const int grid = std::max(1, std::min(ceil_div(n_owned, kWarps), 8 * num_sms()));
  reduce_gather_kernel<<<grid, kWarps * 32, 0, as_stream(stream)>>>(a, n_owned);
  CKV_LAUNCH_CHECK("ckv_reduce_add_gather");
  return CKV_OK;
}

}  // extern "C"
