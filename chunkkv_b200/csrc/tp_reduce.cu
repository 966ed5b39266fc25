// Tensor-parallel exchange over NVLink peer memory, without a collective library:
// the row-parallel GEMM (ckv_linear_push) stores each partial tile straight into the
// receive buffer of the rank that owns its 128-row block; this kernel, on the owning
// rank, sums the ranks' partial rows in a fixed rank order, adds them to the residual
// stream, applies the next RMSNorm, and writes the finished h and x rows to every rank
// (an all-gather by NVLink stores).  Together they replace the NCCL all-reduce after
// o_proj and down_proj (torch_engine.py:70-76 residual adds), with the same result on
// every rank.
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

constexpr int kThreadsRow = 128;
constexpr int kVec = 5;  // 16-byte vectors per thread: hidden <= 128 * 8 * 5 = 5120
constexpr int kRowBlock = 128;

struct ReduceArgs {
  const uint16_t* recv;   // this rank's receive buffer: [ranks][slot] bf16
  int64_t slot;           // elements per source slot
  int rank, ranks;
  int M, hidden;
  uint16_t* h;            // this rank's residual stream [M][hidden] (updated in place)
  uint16_t* x;            // this rank's normed rows [M][hidden]
  const uint16_t* w;      // RMSNorm weight
  float eps;
  const uint64_t* h_peer; // [ranks] h of each rank
  const uint64_t* x_peer; // [ranks] x of each rank
  const unsigned* recv_cnt;    // this rank's receive counters [ranks]
  unsigned* gather_cnt;        // this rank's gather counters [ranks]
  const uint64_t* gather_peer; // [ranks] address of each rank's gather counters
  unsigned* ticket;            // this rank's CTA ticket (left at 0)
  unsigned epoch;              // counters' value once this exchange is complete
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One CTA per owned row.  Owned row i: block rank + (i / 128) * ranks, row i % 128 in it.
__global__ void __launch_bounds__(kThreadsRow) reduce_rmsnorm_kernel(ReduceArgs a) {
  __shared__ float s_red[kThreadsRow / 32];
  __shared__ int s_ok;
  const int i = blockIdx.x;
  const int row = (a.rank + (i / kRowBlock) * a.ranks) * kRowBlock + (i % kRowBlock);
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int q = 0; q < a.ranks && ok; ++q) ok = wait_counter(a.recv_cnt + q, a.epoch, &g_err_word);
    if (!ok) atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  const int vecs = a.hidden / 8;
  if (s_ok && row < a.M) {
    // fixed rank order, fp32: the same bits on every rank
    float acc[kVec][8];
#pragma unroll
    for (int v = 0; v < kVec; ++v)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[v][e] = 0.f;
    for (int q = 0; q < a.ranks; ++q) {
      const uint4* src = reinterpret_cast<const uint4*>(a.recv + q * a.slot + int64_t(row) * a.hidden);
#pragma unroll
      for (int v = 0; v < kVec; ++v) {
        const int c = threadIdx.x + kThreadsRow * v;
        if (c < vecs) {
          const uint4 d = __ldcg(src + c);  // written by other GPUs: not from L1
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(&d);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[v][2 * e] = __fadd_rn(acc[v][2 * e], lo_bf(pw[e]));
            acc[v][2 * e + 1] = __fadd_rn(acc[v][2 * e + 1], hi_bf(pw[e]));
          }
        }
      }
    }
    // h = bf16(h + bf16(sum)), then y = w * bf16(h * rsqrt(mean(h^2) + eps))
    uint4* hr = reinterpret_cast<uint4*>(a.h + int64_t(row) * a.hidden);
    uint4 hv[kVec];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      const int c = threadIdx.x + kThreadsRow * v;
      hv[v] = make_uint4(0u, 0u, 0u, 0u);
      if (c < vecs) {
        const uint4 old = hr[c];
        const uint32_t* po = reinterpret_cast<const uint32_t*>(&old);
        uint32_t* pn = reinterpret_cast<uint32_t*>(&hv[v]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float n0 = __fadd_rn(lo_bf(po[e]), bf16_round(acc[v][2 * e]));
          const float n1 = __fadd_rn(hi_bf(po[e]), bf16_round(acc[v][2 * e + 1]));
          pn[e] = pack_bf2(n0, n1);
          const float f0 = lo_bf(pn[e]), f1 = hi_bf(pn[e]);
          ss = __fadd_rn(ss, __fmul_rn(f0, f0));
          ss = __fadd_rn(ss, __fmul_rn(f1, f1));
        }
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
    __syncthreads();
    const float tot = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
    const float r = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / float(a.hidden)), a.eps));
    const uint4* wr = reinterpret_cast<const uint4*>(a.w);
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      const int c = threadIdx.x + kThreadsRow * v;
      if (c < vecs) {
        const uint4 g = __ldg(wr + c);
        const uint32_t* ph = reinterpret_cast<const uint32_t*>(&hv[v]);
        const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
        uint4 xo;
        uint32_t* px = reinterpret_cast<uint32_t*>(&xo);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float n0 = bf16_round(__fmul_rn(lo_bf(ph[e]), r));
          const float n1 = bf16_round(__fmul_rn(hi_bf(ph[e]), r));
          px[e] = pack_bf2(__fmul_rn(lo_bf(pg[e]), n0), __fmul_rn(hi_bf(pg[e]), n1));
        }
        // every rank's copy of the row, this rank's included
        const int64_t off = int64_t(row) * a.hidden / 8 + c;
        for (int q = 0; q < a.ranks; ++q) {
          reinterpret_cast<uint4*>(a.h_peer[q])[off] = hv[v];
          reinterpret_cast<uint4*>(a.x_peer[q])[off] = xo;
        }
      }
    }
  } else {
    __syncthreads();  // matches the reduction barrier of the rows above
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

int ckv_reduce_add_rmsnorm(const uint16_t* recv, int64_t slot_elems, int rank, int ranks, int m,
                           int hidden, uint16_t* h, uint16_t* x, const uint16_t* w, float eps,
                           const uint64_t* h_peer, const uint64_t* x_peer, const uint32_t* recv_cnt,
                           uint32_t* gather_cnt, const uint64_t* gather_peer, uint32_t* ticket,
                           uint32_t epoch, ckv_stream_t stream) {
  CKV_REQUIRE(recv && h && x && w && h_peer && x_peer && recv_cnt && gather_cnt && gather_peer && ticket,
              "ckv_reduce_add_rmsnorm: null pointer");
  CKV_REQUIRE(ranks >= 1 && ranks <= CKV_MAX_RANKS && rank >= 0 && rank < ranks,
              "ckv_reduce_add_rmsnorm: rank %d of %d", rank, ranks);
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0 && hidden <= kThreadsRow * 8 * kVec,
              "ckv_reduce_add_rmsnorm: hidden %d (multiple of 8, at most %d)", hidden,
              kThreadsRow * 8 * kVec);
  CKV_REQUIRE(aligned16(recv) && aligned16(h) && aligned16(x) && aligned16(w) && slot_elems % 8 == 0 &&
                  slot_elems >= int64_t(m) * hidden,
              "ckv_reduce_add_rmsnorm: alignment or slot size");
  if (m <= 0) return CKV_OK;
  ReduceArgs a{recv, slot_elems, rank, ranks, m, hidden, h, x, w, eps, h_peer, x_peer,
               reinterpret_cast<const unsigned*>(recv_cnt), reinterpret_cast<unsigned*>(gather_cnt),
               gather_peer, reinterpret_cast<unsigned*>(ticket), epoch};
  // every rank launches at least one CTA, so every rank signals its gather counters
  const int grid = std::max(1, owned_rows(m, rank, ranks));
  reduce_rmsnorm_kernel<<<grid, kThreadsRow, 0, as_stream(stream)>>>(a);
  CKV_LAUNCH_CHECK("ckv_reduce_add_rmsnorm");
  return CKV_OK;
}

}  // extern "C"
