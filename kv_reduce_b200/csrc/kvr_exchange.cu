// Cross-GPU exchange + LSE merge of sequence-split decode partials over
// NVLink peer memory (sm_100a), one kernel per decode step.
//
// A sequence split across GPUs leaves every rank with unnormalised partials
// (m, l, o) of its token shard (kvr_decode_partial).  Instead of an all-gather
// collective followed by a merge launch, each rank runs one kernel that
//   1. stores its partials into its slot of every peer's receive buffer
//      (plain st.global through CUDA IPC peer mappings, no TMA, no multicast),
//   2. after a grid-wide arrival count, signals every peer with the step's
//      epoch (system-scope release),
//   3. waits -- bounded in time -- until every peer's epoch has arrived
//      (system-scope acquire), and
//   4. merges all ranks' partials from its own memory into the bf16 output.
// Receive slots alternate between two halves by epoch parity: a peer can be
// one step ahead (it has seen this rank's signal), never two.
//
// Receive buffer of a rank (floats):
//   [2 parities][world sources][rows * (2 + D)]  -- per source: (m, l) pairs
//   [rows][2] then o [rows][D], m in log2 units (kvr_decode_partial's layout)
// followed by a 256-byte signal area: int signal[world] (epoch per source).
#include "kvr_common.cuh"

#include <algorithm>
#include <cstring>

namespace kvr {
namespace xchg {

constexpr int kThreads = 256;
constexpr int kPushCtas = 16;   // CTAs that store to the peers (and fence)

__device__ __forceinline__ void store_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int load_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kThreads) exchange_merge_kernel(kvr_exchange_args a) {
  const int world = a.world, rank = a.rank, rows = a.rows, D = a.head_dim;
  const int e = *reinterpret_cast<volatile int*>(a.epoch) + 1;   // this step's epoch
  const int par = e & 1;
  const int64_t slot = (int64_t)rows * (2 + D);
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gstride = (int64_t)gridDim.x * blockDim.x;

  // 1. push this rank's slot to every peer (the local copy is already in
  //    place).  Only the first kPushCtas CTAs store: a slot is a few hundred
  //    KB, and each storing CTA must wait for its remote stores to land
  //    (a system-scope fence) before it arrives -- with every CTA storing a
  //    sliver, those fences dominated the exchange.
  const int npush = min((int)gridDim.x, kPushCtas);
  if ((int)blockIdx.x < npush) {
    const float* mine = a.recv[rank] + ((int64_t)par * world + rank) * slot;
    const int64_t ptid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t pstride = (int64_t)npush * blockDim.x;
    for (int p = 0; p < world; ++p) {
      if (p == rank) continue;
      float* dst = a.recv[p] + ((int64_t)par * world + rank) * slot;
      if ((slot & 3) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(mine);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (int64_t i = ptid; i < slot / 4; i += pstride) d4[i] = s4[i];
      } else {
        for (int64_t i = ptid; i < slot; i += pstride) dst[i] = mine[i];
      }
    }
  }

  // 2. grid-wide arrival; the last CTA signals every peer
  __syncthreads();
  if (threadIdx.x == 0) {
    if ((int)blockIdx.x < npush) __threadfence_system();   // this CTA's peer stores have landed
    if (atomicAdd(a.counter, 1) == (int)gridDim.x - 1) {
      __threadfence_system();   // every CTA's peer stores precede the signals
      *a.counter = 0;
      for (int p = 0; p < world; ++p)
        if (p != rank) store_release_sys(a.signal[p] + rank, e);
      *a.epoch = e;
    }
  }

  // 3. wait for every peer's epoch (bounded); a time-out is recorded and the
  //    merge then uses whatever is there (the launch's output is invalid)
  if (threadIdx.x == 0) {
    bool ok = true;
    const int* sig = a.signal[rank];
    const uint64_t t0 = global_timer_ns();
    for (int src = 0; src < world && ok; ++src) {
      if (src == rank) continue;
      while (load_acquire_sys(sig + src) < e) {
        if (global_timer_ns() - t0 > (uint64_t)a.timeout_ns) {
          atomicOr(a.error, 1);
          ok = false;
          break;
        }
      }
    }
  }
  __syncthreads();

  // 4. LSE merge of all sources from local memory
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float* base = a.recv[rank] + (int64_t)par * world * slot;
  for (int64_t i = gtid; i < (int64_t)rows * D; i += gstride) {
    const int64_t row = i / D, d = i % D;
    float M = NEG_INF;
    for (int src = 0; src < world; ++src) M = fmaxf(M, base[src * slot + 2 * row]);
    float acc = 0.f, L = 0.f;
    if (M != NEG_INF) {
      for (int src = 0; src < world; ++src) {
        const float* ps = base + src * slot;
        const float m = ps[2 * row];
        if (m == NEG_INF) continue;
        const float w = exp2f(m - M);
        acc = fmaf(w, ps[2 * rows + row * D + d], acc);
        L = fmaf(w, ps[2 * row + 1], L);
      }
    }
    a.out[i] = f32_to_bf16_bits(L > 0.f ? acc / L : 0.f);
  }
}

}  // namespace xchg
}  // namespace kvr

using namespace kvr;

extern "C" int kvr_exchange_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes == 0) return KVR_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    cudaFree(p);
    return KVR_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return KVR_OK;
}

extern "C" int kvr_exchange_open(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) return KVR_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  return KVR_OK;
}

extern "C" int kvr_exchange_close(void* ptr) {
  if (!ptr) return KVR_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  return KVR_OK;
}

extern "C" int kvr_exchange_free(void* ptr) {
  if (!ptr) return KVR_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  return KVR_OK;
}

extern "C" int kvr_exchange_merge(const kvr_exchange_args* a, kvr_stream_t stream) {
  if (!a || a->world < 1 || a->rank < 0 || a->rank >= a->world || a->rows < 1 || a->head_dim < 1 ||
      !a->recv || !a->signal || !a->epoch || !a->counter || !a->out || !a->error || a->timeout_ns <= 0)
    return KVR_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one CTA per SM at most: every CTA is resident while it waits for the peers
  const int64_t work = (int64_t)a->rows * (2 + a->head_dim);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, (work + xchg::kThreads - 1) / xchg::kThreads));
  xchg::exchange_merge_kernel<<<grid, xchg::kThreads, 0, as_stream(stream)>>>(*a);
  return check_launch();
}
