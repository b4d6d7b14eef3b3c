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

// Delivered mode: kvr_decode_partial_exchange has already stored every row
// of this step's partials into each rank's receive area as 8-byte words
// (value, epoch), each written whole -- the low-latency protocol NCCL
// publishes as "LL".  Nothing is pushed or fenced here: one warp per row
// reads every source's words for the row until all of them carry this
// step's epoch (bounded by the launch's deadline), then merges the row.
// The last CTA to finish advances the epoch.
constexpr int kLLWords = 64;   // receive area: 32-bit words after the signal words

__device__ __forceinline__ uint4 ld_volatile_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

// Merge of one row from the tagged words of every source at `area` (layout
// [world sources][rows][2 + D][2] words): every source's (m, l) words and
// this lane's four o words, all loads in flight at once; then only the words
// whose tag is not yet e are read again, until the deadline (then
// *timed_out is set and what is there is merged).  Returns this lane's four
// bf16 outputs (d = 4 * lane) as two words, acc / L as in kvr_lse_merge, so
// the two merges agree bit for bit.
__device__ __forceinline__ uint2 merge_row(const uint32_t* area, int64_t lslot, int world, int row, int D,
                                           uint32_t e, uint64_t deadline, bool* timed_out) {
  const int lane = threadIdx.x & 31;
  const int d = 4 * lane;
  const bool dl = d < D;
  const float NEG_INF = -__int_as_float(0x7f800000);
  uint4 wml[8], wo0[8], wo1[8];
  const uint4 zero = make_uint4(0u, e, 0u, e);
#pragma unroll
  for (int src = 0; src < 8; ++src) {
    const uint32_t* r = area + src * lslot + (int64_t)row * (2 + D) * 2;
    wml[src] = src < world ? ld_volatile_v4(r) : zero;
    wo0[src] = (src < world && dl) ? ld_volatile_v4(r + 2 * (2 + d)) : zero;
    wo1[src] = (src < world && dl) ? ld_volatile_v4(r + 2 * (2 + d) + 4) : zero;
  }
  for (;;) {
    bool ready = true;
#pragma unroll
    for (int src = 0; src < 8; ++src) {
      if (src >= world) break;
      const uint32_t* r = area + src * lslot + (int64_t)row * (2 + D) * 2;
      if (wml[src].y != e || wml[src].w != e) { ready = false; wml[src] = ld_volatile_v4(r); }
      if (wo0[src].y != e || wo0[src].w != e) { ready = false; wo0[src] = ld_volatile_v4(r + 2 * (2 + d)); }
      if (wo1[src].y != e || wo1[src].w != e) { ready = false; wo1[src] = ld_volatile_v4(r + 2 * (2 + d) + 4); }
    }
    if (ready || *timed_out) break;
    if (global_timer_ns() > deadline) *timed_out = true;   // one more pass, then merge what is there
  }
  float M = NEG_INF;
#pragma unroll
  for (int src = 0; src < 8; ++src)
    if (src < world) M = fmaxf(M, __uint_as_float(wml[src].x));
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.f;
#pragma unroll
  for (int src = 0; src < 8; ++src) {
    if (src >= world) break;
    const float m = __uint_as_float(wml[src].x);
    if (M == NEG_INF || m == NEG_INF) continue;
    const float wt = exp2f(m - M);
    acc.x = fmaf(wt, __uint_as_float(wo0[src].x), acc.x); acc.y = fmaf(wt, __uint_as_float(wo0[src].z), acc.y);
    acc.z = fmaf(wt, __uint_as_float(wo1[src].x), acc.z); acc.w = fmaf(wt, __uint_as_float(wo1[src].z), acc.w);
    L = fmaf(wt, __uint_as_float(wml[src].z), L);
  }
  const bool nz = L > 0.f;
  uint2 pk;
  pk.x = (uint32_t)f32_to_bf16_bits(nz ? acc.x / L : 0.f) | ((uint32_t)f32_to_bf16_bits(nz ? acc.y / L : 0.f) << 16);
  pk.y = (uint32_t)f32_to_bf16_bits(nz ? acc.z / L : 0.f) | ((uint32_t)f32_to_bf16_bits(nz ? acc.w / L : 0.f) << 16);
  return pk;
}

// The last CTA to arrive advances the epoch (every CTA read it first).
__device__ __forceinline__ void advance_epoch(const kvr_exchange_args& a, int ep) {
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.counter, 1) == (int)gridDim.x - 1) {
    *a.counter = 0;
    *a.epoch = ep;
  }
}

__global__ void __launch_bounds__(kThreads) merge_delivered_kernel(kvr_exchange_args a) {
  // launched as a programmatic dependent of this rank's decode: resident
  // early, but nothing is read before that decode has completed
  pdl_wait();
  const int world = a.world, rank = a.rank, rows = a.rows, D = a.head_dim;
  const int ep = *reinterpret_cast<volatile int*>(a.epoch) + 1;
  const int64_t lslot = (int64_t)rows * (2 + D) * 2;   // words per (half, source)
  const uint32_t* area = reinterpret_cast<const uint32_t*>(a.signal[rank]) + kLLWords + (int64_t)(ep & 1) * world * lslot;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int d = 4 * lane;
  const uint64_t deadline = global_timer_ns() + (uint64_t)a.timeout_ns;
  bool timed_out = false;
  for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
    const uint2 pk = merge_row(area, lslot, world, row, D, (uint32_t)ep, deadline, &timed_out);
    if (d < D) *reinterpret_cast<uint2*>(a.out + (int64_t)row * D + d) = pk;
  }
  if (timed_out) atomicOr(a.error, 1);   // some row merged whatever was there: the output is invalid
  advance_epoch(a, ep);
}

// Owner mode, first kernel: the rows this rank owns (row % world == rank)
// arrived from every rank (kvr_decode_partial_exchange with mode 1); merge
// each, write it to out and store it, as tagged words (bf16 pair, epoch),
// into every peer's final area: words [2 halves][rows][D] after the receive
// area, a lane's four outputs as one 16-byte store.
__global__ void __launch_bounds__(kThreads) merge_owned_kernel(kvr_exchange_args a) {
  pdl_wait();
  const int world = a.world, rank = a.rank, rows = a.rows, D = a.head_dim;
  const int ep = *reinterpret_cast<volatile int*>(a.epoch) + 1;
  const uint32_t e = (uint32_t)ep;
  const int64_t lslot = (int64_t)rows * (2 + D) * 2;
  const uint32_t* area = reinterpret_cast<const uint32_t*>(a.signal[rank]) + kLLWords + (int64_t)(ep & 1) * world * lslot;
  const int64_t final_off = kLLWords + 2 * (int64_t)world * lslot + (int64_t)(ep & 1) * rows * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int d = 4 * lane;
  const int n_own = (rows - rank + world - 1) / world;
  const uint64_t deadline = global_timer_ns() + (uint64_t)a.timeout_ns;
  bool timed_out = false;
  for (int j = blockIdx.x * warps + warp; j < n_own; j += gridDim.x * warps) {
    const int row = rank + j * world;
    const uint2 pk = merge_row(area, lslot, world, row, D, e, deadline, &timed_out);
    if (d < D) {
      *reinterpret_cast<uint2*>(a.out + (int64_t)row * D + d) = pk;
      for (int r = 0; r < world; ++r) {
        if (r == rank) continue;
        uint32_t* f = reinterpret_cast<uint32_t*>(a.signal[r]) + final_off + (int64_t)row * D + d;
        asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"l"(f), "r"(pk.x), "r"(e), "r"(pk.y),
                     "r"(e) : "memory");
      }
    }
  }
  if (timed_out) atomicOr(a.error, 1);
}

// Owner mode, second kernel: the rows other ranks own, read from this rank's
// final area until every word carries this step's epoch (bounded), into
// out; the last CTA advances the epoch.
__global__ void __launch_bounds__(kThreads) gather_owned_kernel(kvr_exchange_args a) {
  pdl_wait();
  const int world = a.world, rank = a.rank, rows = a.rows, D = a.head_dim;
  const int ep = *reinterpret_cast<volatile int*>(a.epoch) + 1;
  const uint32_t e = (uint32_t)ep;
  const int64_t lslot = (int64_t)rows * (2 + D) * 2;
  const uint32_t* fin = reinterpret_cast<const uint32_t*>(a.signal[rank]) + kLLWords + 2 * (int64_t)world * lslot +
                        (int64_t)(ep & 1) * rows * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int d = 4 * lane;
  const uint64_t deadline = global_timer_ns() + (uint64_t)a.timeout_ns;
  bool timed_out = false;
  for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
    if (row % world == rank || d >= D) continue;   // owned rows were written by merge_owned_kernel
    const uint32_t* f = fin + (int64_t)row * D + d;
    uint4 v = ld_volatile_v4(f);
    while ((v.y != e || v.w != e) && !timed_out) {
      if (global_timer_ns() > deadline) timed_out = true;
      v = ld_volatile_v4(f);
    }
    *reinterpret_cast<uint2*>(a.out + (int64_t)row * D + d) = make_uint2(v.x, v.z);
  }
  if (timed_out) atomicOr(a.error, 1);
  advance_epoch(a, ep);
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

extern "C" int kvr_exchange_merge_delivered(const kvr_exchange_args* a, kvr_stream_t stream) {
  if (!a || a->world < 1 || a->world > 8 || a->rank < 0 || a->rank >= a->world || a->rows < 1 ||
      (a->head_dim != 64 && a->head_dim != 128) || !a->signal || !a->epoch || !a->counter || !a->out ||
      !a->error || a->timeout_ns <= 0)
    return KVR_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one warp per row, one CTA per SM at most: every CTA is resident while it waits
  constexpr int warps = xchg::kThreads / 32;
  const int grid = std::max(1, std::min(sms, (a->rows + warps - 1) / warps));
  (void)pdl_launch(xchg::merge_delivered_kernel, dim3(grid), dim3(xchg::kThreads), 0, as_stream(stream), 1, *a);
  return check_launch();
}

static int check_owner_args(const kvr_exchange_args* a) {
  if (!a || a->world < 1 || a->world > 8 || a->rank < 0 || a->rank >= a->world || a->rows < 1 ||
      (a->head_dim != 64 && a->head_dim != 128) || !a->signal || !a->epoch || !a->counter || !a->out ||
      !a->error || a->timeout_ns <= 0)
    return KVR_ERR_INVALID_ARGUMENT;
  return KVR_OK;
}

extern "C" int kvr_exchange_merge_owned(const kvr_exchange_args* a, kvr_stream_t stream) {
  const int st = check_owner_args(a);
  if (st != KVR_OK) return st;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int warps = xchg::kThreads / 32;
  const int n_own = (a->rows - a->rank + a->world - 1) / a->world;
  const int grid = std::max(1, std::min(sms, (n_own + warps - 1) / warps));
  (void)pdl_launch(xchg::merge_owned_kernel, dim3(grid), dim3(xchg::kThreads), 0, as_stream(stream), 1, *a);
  return check_launch();
}

extern "C" int kvr_exchange_gather_owned(const kvr_exchange_args* a, kvr_stream_t stream) {
  const int st = check_owner_args(a);
  if (st != KVR_OK) return st;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int warps = xchg::kThreads / 32;
  const int grid = std::max(1, std::min(sms, (a->rows + warps - 1) / warps));
  (void)pdl_launch(xchg::gather_owned_kernel, dim3(grid), dim3(xchg::kThreads), 0, as_stream(stream), 1, *a);
  return check_launch();
}
