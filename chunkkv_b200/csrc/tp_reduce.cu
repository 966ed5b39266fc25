// Tensor-parallel exchange over NVLink peer memory, without a collective library:
// every rank's row-parallel GEMM (ckv_linear_partial) writes its partial rows into its
// own buffer and signals; this kernel, on the rank that owns a 128-row block (block b ->
// rank b % ranks), copies the ranks' partial rows of that block over NVLink (TMA bulk
// copies of whole row segments), sums them in a fixed rank order, adds them to the
// residual stream, and writes the finished h rows to every rank (an all-gather by bulk
// stores over NVLink).  Together they replace the NCCL all-reduce after o_proj and down_proj
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

// Bounded wait that ignores any abort flag (used only while draining).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitLimitNs) break;
}

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

// The rows move by TMA bulk copies, whole contiguous row segments at a time: a unit is
// (owned row, segment of seg_cols(T, hidden) columns); for each unit one thread copies the
// T ranks' partial segments from their buffers (over NVLink, plain peer loads) into
// shared memory, completing on the stage's mbarrier; all threads then sum them in rank
// order and add the residual into an output segment in shared memory, which one thread
// stores into every rank's h (bulk stores to peer memory).  Two stages per CTA, so the
// next unit's copies are in flight while this one is summed.  (Per-lane 16-byte loads
// and stores of the same rows reached about 60 % of the NVLink bandwidth.)
constexpr int kThreads = 256;
constexpr int kStages = 2;
constexpr int kSmemBudget = 200 * 1024;  // dynamic shared memory per CTA, both stages
// columns per unit for T ranks: (T + 1) segments (T inputs, one output) per stage
__host__ __device__ inline int seg_cols(int T, int hidden) {
  int w = kSmemBudget / (kStages * (T + 1) * 2);
  w = w / 8 * 8;
  return hidden < w ? hidden : w;
}

template <int T>
__global__ void __launch_bounds__(kThreads, 1) reduce_gather_kernel(ReduceArgs a, int n_owned) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ int s_ok;
  const int W = seg_cols(T, a.hidden);           // columns per unit
  const int segs = (a.hidden + W - 1) / W;
  const int units = n_owned * segs;
  const int64_t stage_elems = int64_t(T + 1) * W;  // bf16 elements per stage
  uint16_t* sm = reinterpret_cast<uint16_t*>(smem);
  auto unit_row = [&](int u, int& row, int& c0, int& cols) {
    const int i = u / segs, sg = u - (u / segs) * segs;
    row = (a.rank + (i / kRowBlock) * a.ranks) * kRowBlock + (i % kRowBlock);
    c0 = sg * W;
    cols = min(W, a.hidden - c0);
  };
  // copies of the k-th unit of this CTA into stage k % 2 (thread 0)
  auto issue_loads = [&](int k) {
    const int u = blockIdx.x + k * gridDim.x;
    int row, c0, cols;
    unit_row(u, row, c0, cols);
    uint64_t* bar = &full[k & 1];
    const uint32_t bytes = uint32_t(cols) * 2;
    mbar_expect_tx(bar, bytes * T);
    uint16_t* st = sm + (k & 1) * stage_elems;
#pragma unroll
    for (int q = 0; q < T; ++q)
      bulk_load(st + int64_t(q) * W, reinterpret_cast<const uint16_t*>(a.part[q]) + int64_t(row) * a.hidden + c0,
                bytes, bar);
  };
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    bool ok = true;
    for (int q = 0; q < a.ranks && ok; ++q) ok = wait_counter(a.recv_cnt + q, a.epoch, &g_err_word);
    if (!ok) atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
    s_ok = ok;
    // the partial rows are final on every rank: start the first two units' copies (the
    // proxy fence orders the acquire above before the copy engine's reads)
    asm volatile("fence.proxy.async.global;" ::: "memory");
    if (ok)
      for (int k = 0; k < kStages && k < my_units; ++k) issue_loads(k);
  }
  __syncthreads();
  if (s_ok) {
    volatile int no_abort = 0;
    for (int k = 0; k < my_units; ++k) {
      const int st_i = k & 1;
      int row, c0, cols;
      unit_row(blockIdx.x + k * gridDim.x, row, c0, cols);
      uint16_t* in = sm + st_i * stage_elems;
      uint16_t* out = in + int64_t(T) * W;
      if (threadIdx.x == 0) {
        // the stores of unit k - 2 have read this stage's output segment
        if (k >= kStages) bulk_wait_read<kStages - 1>();
        // this unit's copies have landed (bounded; thread 0 waits, the barrier below
        // hands the data to the other threads)
        if (!mbar_wait(&full[st_i], (k / kStages) & 1, &no_abort, &g_err_word)) {
          atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
          s_ok = 0;
          // let the copies already issued (this unit's and the next one's) land
          // before the CTA's shared memory goes away
          for (int j = k; j < k + kStages && j < my_units; ++j) drain_wait(&full[j & 1], (j / kStages) & 1);
        }
      }
      __syncthreads();
      if (!s_ok) break;
      const int vecs = cols / 8;
      const uint4* h_old = reinterpret_cast<const uint4*>(a.h + int64_t(row) * a.hidden + c0);
      for (int v = threadIdx.x; v < vecs; v += kThreads) {
        // fixed rank order, fp32: the same bits on every rank; then h = bf16(h + bf16(sum))
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
        for (int q = 0; q < T; ++q) {
          const uint4 d = reinterpret_cast<const uint4*>(in + int64_t(q) * W)[v];
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(&d);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] = __fadd_rn(acc[2 * e], lo_bf(pw[e]));
            acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], hi_bf(pw[e]));
          }
        }
        const uint4 old = h_old[v];
        const uint32_t* po = reinterpret_cast<const uint32_t*>(&old);
        uint4 hv;
        uint32_t* pn = reinterpret_cast<uint32_t*>(&hv);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pn[e] = pack_bf2(__fadd_rn(lo_bf(po[e]), bf16_round(acc[2 * e])),
                           __fadd_rn(hi_bf(po[e]), bf16_round(acc[2 * e + 1])));
        reinterpret_cast<uint4*>(out)[v] = hv;
      }
      fence_async_smem();
      __syncthreads();  // the output segment is written and this stage's inputs are read
      if (threadIdx.x == 0) {
        // the finished segment into every rank's h (this rank's own included)
#pragma unroll
        for (int q = 0; q < T; ++q)
          bulk_store(reinterpret_cast<uint16_t*>(a.h_peer[q]) + int64_t(row) * a.hidden + c0, out,
                     uint32_t(cols) * 2);
        bulk_commit();
        if (k + kStages < my_units) issue_loads(k + kStages);
      }
    }
  }
  if (threadIdx.x == 0) {
    bulk_wait_all();  // the h stores have been written
    asm volatile("fence.proxy.async.global;" ::: "memory");
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
  cudaStream_t s = as_stream(stream);
  auto go = [&](auto kern, int T) -> int {
    const int W = seg_cols(T, hidden);
    const int units = n_owned * ceil_div(hidden, W);
    const int smem = kStages * (T + 1) * W * 2;
    if (int rc = set_smem_limit(reinterpret_cast<const void*>(kern), smem)) return rc;
    // one CTA per SM at most (each holds both stages); every rank launches at least one
    // CTA, so every rank signals its gather counters
    const int grid = std::max(1, std::min(units, num_sms()));
    kern<<<grid, kThreads, smem, s>>>(a, n_owned);
    return CKV_OK;
  };
  int rc;
  switch (ranks) {
    case 1: rc = go(reduce_gather_kernel<1>, 1); break;
    case 2: rc = go(reduce_gather_kernel<2>, 2); break;
    case 4: rc = go(reduce_gather_kernel<4>, 4); break;
    case 8: rc = go(reduce_gather_kernel<8>, 8); break;
    default:
      set_error("ckv_reduce_add_gather: %d ranks (1, 2, 4 or 8)", ranks);
      return CKV_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  CKV_LAUNCH_CHECK("ckv_reduce_add_gather");
  return CKV_OK;
}

}  // extern "C"
