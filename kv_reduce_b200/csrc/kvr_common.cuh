// Shared helpers for the packed draft-KV kernels (sm_100a).
//
// Never compile this project with --use_fast_math: the quantizer must
// reproduce IEEE fp32 division and round-half-even exactly as
// kv_reduce/packed_kv_cache.py:181-182 / :240-241 does through torch.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kvr.h"

namespace kvr {

// ----------------------------------------------------------------- status
// Records the CUDA error text of the last failing call on this host thread.
void set_last_cuda_error(cudaError_t e);

inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  return KVR_OK;
}

inline cudaStream_t as_stream(kvr_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------- programmatic dependent launch
// The decode and append kernels of a decode loop are launched with
// programmatic stream serialization (pdl_launch): the next such kernel in the
// stream may be scheduled while this one still runs.  Each of them calls
// pdl_wait() before touching global memory: it waits until the previous
// kernel in the stream has completed and its memory operations are visible
// -- so the ordering is the stream's, and only the launch latency overlaps.
// pdl_trigger() lets the next kernel be scheduled: at the start of a short
// kernel (pdl_enter), after its main loop for a long one, so the next
// kernel's CTAs are not placed beside a running wave.  A previous kernel that never
// triggers (any other code's kernel) simply completes first.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_trigger();
  pdl_wait();
}

template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ------------------------------------------------------------ bf16 bits
// bf16 <-> fp32 on raw 16-bit patterns.  bf16 -> fp32 is exact; fp32 ->
// bf16 rounds to nearest even like torch's Tensor.to(torch.bfloat16).
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
// Low / high bf16 of a packed 32-bit word as fp32.
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ------------------------------------------------------------ quantizer
// scale = max(max-min, 1e-8) / (2^bits-1), IEEE division
// (packed_kv_cache.py:181 and :240).
__device__ __forceinline__ float affine_scale(float mn, float mx, int bits) {
  float range = __fsub_rn(mx, mn);
  range = fmaxf(range, 1e-8f);
  return __fdiv_rn(range, static_cast<float>((1 << bits) - 1));
}
// code = clamp(round_half_even((x - min) / scale), 0, 2^bits-1)
// (packed_kv_cache.py:182 and :241).
__device__ __forceinline__ uint32_t affine_code(float x, float mn, float scale, int bits) {
  float q = rintf(__fdiv_rn(__fsub_rn(x, mn), scale));
  q = fminf(fmaxf(q, 0.0f), static_cast<float>((1 << bits) - 1));
  return static_cast<uint32_t>(q);
}
// dequant = code * scale + offset with two roundings, no FMA contraction
// (packed_kv_cache.py:131 and :145).
__device__ __forceinline__ float affine_dequant(uint32_t code, float scale, float offset) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), scale), offset);
}

// Exact affine code with a reciprocal.  q = fl(x - mn) * fl(1/scale) is
// within 1.5 * 2^-23 * q of the reference's quotient fl(fl(x - mn) / scale)
// (< 5e-5 for codes up to 255), so both round to the same integer unless q
// lies within that distance of n + 0.5; within 1e-3 of it the exact IEEE
// division decides.
static __device__ __noinline__ float exact_quotient(float diff, float scale) { return __fdiv_rn(diff, scale); }

static __device__ __forceinline__ uint32_t affine_code_rcp(float x, float mn, float scale, float inv, int levels) {
  const float diff = __fsub_rn(x, mn);
  float q = __fmul_rn(diff, inv);
  float r = rintf(q);
  if (fabsf(q - r) > 0.5f - 1e-3f) r = rintf(exact_quotient(diff, scale));   // near n + 0.5: rare
  r = fminf(fmaxf(r, 0.f), (float)levels);
  return (uint32_t)r;
}

// N bf16 values (N in {2, 4, 8}) as fp32, from one vector load.
template <int N>
static __device__ __forceinline__ void load_bf16x(const uint16_t* p, float (&v)[N]) {
  uint32_t w[N / 2];
  if constexpr (N == 2) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (N == 4) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    w[0] = x.x; w[1] = x.y;
  } else {
    const uint4 x = *reinterpret_cast<const uint4*>(p);
    w[0] = x.x; w[1] = x.y; w[2] = x.z; w[3] = x.w;
  }
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    v[2 * i] = bf16lo(w[i]);
    v[2 * i + 1] = bf16hi(w[i]);
  }
}

// Store the low NB bytes of `w` (NB in {1, 2, 4, 8}).
template <int NB>
static __device__ __forceinline__ void store_bytes(uint8_t* p, uint64_t w) {
  if constexpr (NB == 1) *p = (uint8_t)w;
  else if constexpr (NB == 2) *reinterpret_cast<uint16_t*>(p) = (uint16_t)w;
  else if constexpr (NB == 4) *reinterpret_cast<uint32_t*>(p) = (uint32_t)w;
  else *reinterpret_cast<uint2*>(p) = make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}


// Byte `byte_idx` of the LSB-first bitstream of `codes` (bits per code),
// reading codes from `get(i)` for i in [0, n).  Works for any bits in 1..8.
template <typename Get>
__device__ __forceinline__ uint32_t stream_byte(int64_t byte_idx, int bits, int64_t n, Get get) {
  const int64_t bit0 = byte_idx * 8;
  int64_t i = bit0 / bits;
  const int64_t bit_end = bit0 + 8;
  uint32_t out = 0;
  for (; i < n && i * bits < bit_end; ++i) {
    const int64_t pos = i * bits - bit0;  // may be negative for the first code
    uint32_t c = get(i) & ((1u << bits) - 1u);
    if (pos >= 0) out |= c << pos;
    else out |= c >> (-pos);
  }
  return out & 0xffu;
}

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t x, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (x & mask) | orv  -> lop3 immediate 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(x), "r"(mask), "r"(orv));
  return r;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(r) : "r"(x));
  return r;
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Same with bf16 inputs (BF16 residual keys x BF16 query: exact products).
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x with the hardware approximation (ex2.approx.ftz: ~2 ulp; inputs here
// are x <= 0 from the online softmax, tiny results flush to zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Exact product split in fp16x2 (TwoProduct with a fused multiply-add):
// hi = fl(a*b), lo = fma(a, b, -hi); hi + lo == a*b exactly unless the
// error term falls into the fp16 subnormal range.  -hi is a floating-point
// negate, which the compiler folds into the fma's operand.
__device__ __forceinline__ void two_prod_h2(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(hi) : "r"(a), "r"(b));
  uint32_t nhi;
  asm("neg.f16x2 %0, %1;\n" : "=r"(nhi) : "r"(hi));
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(lo) : "r"(a), "r"(b), "r"(nhi));
}

}  // namespace kvr
