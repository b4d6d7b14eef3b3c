// Quantize-and-pack, unpack and streaming-cache kernels for the packed
// draft-KV cache (sm_100a).
//
// Bit-exactness contract with kv_reduce/packed_kv_cache.py:
//   * statistics on x.float() (exact), scale = max(max-min,1e-8)/(2^b-1)
//     by IEEE division, code = rint((x-min)/scale) clamped   (:179-182, :238-241)
//   * metadata stored as bf16 (round to nearest even)          (:185-186, :244-245)
//   * codes packed LSB-first into a flat byte stream           (:28-63)
// These kernels are HBM-bound byte work: one warp per token row (values) or
// one thread per channel of a key group (keys), codes staged in shared
// memory, bytes emitted by whole warps so stores stay coalesced.
#include "kvr_common.cuh"

#include <algorithm>

namespace kvr {

// ================================================================ primitives
// pack_unsigned (packed_kv_cache.py:28-63): one thread per output byte.
__global__ void pack_unsigned_kernel(const uint8_t* __restrict__ codes, int64_t n, int bits,
                                     uint8_t* __restrict__ payload, int64_t nbytes) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nbytes;
       b += (int64_t)gridDim.x * blockDim.x) {
    payload[b] = (uint8_t)stream_byte(b, bits, n, [&](int64_t i) { return (uint32_t)codes[i]; });
  }
}

// unpack_unsigned (packed_kv_cache.py:66-94): one thread per code.
__global__ void unpack_unsigned_kernel(const uint8_t* __restrict__ payload, int64_t nbytes,
                                       int64_t n, int bits, uint8_t* __restrict__ codes) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bit = i * bits;
    const int64_t byte = bit >> 3;
    const int off = (int)(bit & 7);
    uint32_t w = payload[byte];
    if (off + bits > 8 && byte + 1 < nbytes) w |= (uint32_t)payload[byte + 1] << 8;
    codes[i] = (uint8_t)((w >> off) & ((1u << bits) - 1u));
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  g = std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32));
  return (int)g;
}

// ========================================================= per-token values
// One warp per (bh, row).  Row bytes are emitted from the shared code row.
// `generic` (rows not byte-aligned): codes go to `scratch` (flat index
// (bh*rows + r)*D + d) and a second pass packs the whole stream.
constexpr int kTokWarps = 8;
constexpr int kMaxD = 256;

__global__ void __launch_bounds__(kTokWarps * 32)
quant_token_kernel(kvr_token_quant_args a, int generic) {
  __shared__ uint8_t codes_s[kTokWarps][kMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = (int64_t)a.bh * a.rows;
  const int D = a.head_dim, bits = a.bits;
  const int64_t row_bytes = (int64_t)D * bits / 8;
  for (int64_t item = (int64_t)blockIdx.x * kTokWarps + warp; item < total;
       item += (int64_t)gridDim.x * kTokWarps) {
    const int64_t bh = item / a.rows;
    const int r = (int)(item % a.rows);
    const uint16_t* x = a.x + bh * a.x_bh_stride + (int64_t)r * a.x_row_stride;
    float xv[kMaxD / 32];
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) {
      const int d = lane + 32 * k;
      xv[k] = 0.f;
      if (d < D) {
        xv[k] = bf16_bits_to_f32(x[d]);
        mn = fminf(mn, xv[k]);
        mx = fmaxf(mx, xv[k]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = affine_scale(mn, mx, bits);
    const int64_t meta = bh * a.meta_bh_stride + a.row0 + r;
    if (lane == 0) {
      a.scale[meta] = f32_to_bf16_bits(scale);
      a.offset[meta] = f32_to_bf16_bits(mn);
    }
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) {
      const int d = lane + 32 * k;
      if (d < D) {
        const uint8_t c = (uint8_t)affine_code(xv[k], mn, scale, bits);
        if (generic) a.codes_scratch[(bh * a.rows + r) * (int64_t)D + d] = c;
        else codes_s[warp][d] = c;
      }
    }
    if (!generic) {
      __syncwarp();
      uint8_t* dst = a.payload + bh * a.payload_bh_stride + (int64_t)(a.row0 + r) * row_bytes;
      for (int64_t b = lane; b < row_bytes; b += 32)
        dst[b] = (uint8_t)stream_byte(b, bits, D, [&](int64_t i) { return (uint32_t)codes_s[warp][i]; });
      __syncwarp();
    }
  }
}

// ===================================================== grouped per-channel keys
// One CTA per (bh, group); thread d owns channel d: min/max over the G
// tokens of the group, codes to shared memory, then the CTA emits the G
// payload rows.  Codes in shared memory: [G][D] bytes.
__global__ void quant_group_kernel(kvr_group_quant_args a, int generic) {
  extern __shared__ uint8_t codes_s[];
  const int D = a.head_dim, G = a.group_size, bits = a.bits;
  const int64_t row_bytes = (int64_t)D * bits / 8;
  const int64_t total = (int64_t)a.bh * a.groups;
  for (int64_t item = blockIdx.x; item < total; item += gridDim.x) {
    const int64_t bh = item / a.groups;
    const int gi = (int)(item % a.groups);
    const int g = a.group0 + gi;
    const uint16_t* x = a.x + bh * a.x_bh_stride + (int64_t)gi * G * a.x_row_stride;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
      for (int t = 0; t < G; ++t) {
        const float v = bf16_bits_to_f32(x[(int64_t)t * a.x_row_stride + d]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
      const float scale = affine_scale(mn, mx, bits);
      const int64_t meta = bh * a.meta_bh_stride + (int64_t)g * D + d;
      a.scale[meta] = f32_to_bf16_bits(scale);
      a.offset[meta] = f32_to_bf16_bits(mn);
      for (int t = 0; t < G; ++t) {
        const float v = bf16_bits_to_f32(x[(int64_t)t * a.x_row_stride + d]);
        const uint8_t c = (uint8_t)affine_code(v, mn, scale, bits);
        if (generic) {
          // flat code index of the reference layout [BH, P, D]
          const int64_t rows_per_slab = (int64_t)(a.group0 + a.groups) * G;
          a.codes_scratch[(bh * rows_per_slab + (int64_t)g * G + t) * D + d] = c;
        } else {
          codes_s[t * D + d] = c;
        }
      }
    }
    if (!generic) {
      __syncthreads();
      uint8_t* dst = a.payload + bh * a.payload_bh_stride + (int64_t)g * G * row_bytes;
      const int64_t nb = (int64_t)G * row_bytes;
      for (int64_t b = threadIdx.x; b < nb; b += blockDim.x) {
        const int t = (int)(b / row_bytes);
        const int64_t rb = b - (int64_t)t * row_bytes;
        const uint8_t* crow = codes_s + t * D;
        dst[b] = (uint8_t)stream_byte(rb, bits, D, [&](int64_t i) { return (uint32_t)crow[i]; });
      }
      __syncthreads();
    }
  }
}

// ================================================================ dequantize
// One thread per output element.  Code extraction from the flat bit
// position, so both byte-aligned rows and the reference's flat stream for
// odd shapes are read correctly.
__global__ void dequant_kernel(kvr_dequant_args a, int flat_stream) {
  const int D = a.head_dim, bits = a.bits, S = a.seq_len;
  const bool keys = a.group_size > 0;
  const int P = keys ? a.prefix_len : S;
  const int64_t row_bytes_num = (int64_t)D * bits;  // bits per row
  const int64_t total = (int64_t)a.bh * S * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int64_t rowi = i / D;
    const int t = (int)(rowi % S);
    const int64_t bh = rowi / S;
    float v;
    if (t < P) {
      int64_t bit;
      if (flat_stream) bit = ((bh * P + t) * (int64_t)D + d) * bits;
      else bit = (bh * a.payload_bh_stride) * 8 + (int64_t)t * row_bytes_num + (int64_t)d * bits;
      const int64_t byte = bit >> 3;
      const int off = (int)(bit & 7);
      uint32_t w = a.payload[byte];
      if (off + bits > 8) w |= (uint32_t)a.payload[byte + 1] << 8;
      const uint32_t code = (w >> off) & ((1u << bits) - 1u);
      int64_t meta;
      if (keys) meta = bh * a.meta_bh_stride + (int64_t)(t / a.group_size) * D + d;
      else meta = bh * a.meta_bh_stride + t;
      v = affine_dequant(code, bf16_bits_to_f32(a.scale[meta]), bf16_bits_to_f32(a.offset[meta]));
    } else {
      v = bf16_bits_to_f32(a.residual[bh * a.residual_bh_stride + (int64_t)(t - P) * D + d]);
    }
    if (a.out_dtype == 1) static_cast<float*>(a.out)[i] = v;
    else if (a.out_dtype == 2) static_cast<__half*>(a.out)[i] = __float2half_rn(v);
    else static_cast<uint16_t*>(a.out)[i] = f32_to_bf16_bits(v);
  }
}

// ============================================================ streaming cache
// Append: warp per (bh, new token).  Key row copied into the BF16 residual
// window; value row quantized per token at row seq_len + i.
__global__ void __launch_bounds__(kTokWarps * 32) append_kernel(kvr_append_args a, int* lengths) {
  __shared__ uint8_t codes_s[kTokWarps][kMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.head_dim, bits = a.value_bits;
  if (lengths) {
    // positions from device memory (graph-replayable loops); a step past
    // either capacity sets the error flag lengths[2] and writes nothing
    const int S = *reinterpret_cast<volatile int*>(lengths);
    const int P = *reinterpret_cast<volatile int*>(lengths + 1);
    if (P < 0 || P > S || S + a.n > a.seq_capacity || S - P + a.n > a.res_capacity) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(lengths + 2, 1);
      return;
    }
    a.seq_len = S;
    a.res_len = S - P;
  }
  const int64_t row_bytes = (int64_t)D * bits / 8;
  const int64_t total = (int64_t)a.bh * a.n;
  for (int64_t item = (int64_t)blockIdx.x * kTokWarps + warp; item < total;
       item += (int64_t)gridDim.x * kTokWarps) {
    const int64_t bh = item / a.n;
    const int i = (int)(item % a.n);
    const uint16_t* k = a.k + item * D;
    const uint16_t* v = a.v + item * D;
    uint16_t* kr = a.key_residual + bh * a.key_residual_bh_stride + (int64_t)(a.res_len + i) * D;
    for (int d = lane; d < D; d += 32) kr[d] = k[d];
    float xv[kMaxD / 32];
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int kk = 0; kk < kMaxD / 32; ++kk) {
      const int d = lane + 32 * kk;
      xv[kk] = 0.f;
      if (d < D) {
        xv[kk] = bf16_bits_to_f32(v[d]);
        mn = fminf(mn, xv[kk]);
        mx = fmaxf(mx, xv[kk]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = affine_scale(mn, mx, bits);
    const int64_t meta = bh * a.value_meta_bh_stride + a.seq_len + i;
    if (lane == 0) {
      a.value_scale[meta] = f32_to_bf16_bits(scale);
      a.value_offset[meta] = f32_to_bf16_bits(mn);
    }
#pragma unroll
    for (int kk = 0; kk < kMaxD / 32; ++kk) {
      const int d = lane + 32 * kk;
      if (d < D) codes_s[warp][d] = (uint8_t)affine_code(xv[kk], mn, scale, bits);
    }
    __syncwarp();
    uint8_t* dst = a.value_payload + bh * a.value_payload_bh_stride + (int64_t)(a.seq_len + i) * row_bytes;
    for (int64_t b = lane; b < row_bytes; b += 32)
      dst[b] = (uint8_t)stream_byte(b, bits, D, [&](int64_t j) { return (uint32_t)codes_s[warp][j]; });
    __syncwarp();
  }
}

// Residual window shift after a flush: rows [shift, res_len) -> [0, ..).
__global__ void residual_move_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                     int64_t bh_stride, int bh, int shift, int keep, int D) {
  const int64_t per = (int64_t)keep * D;
  const int64_t total = (int64_t)bh * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per, r = i % per;
    dst[b * bh_stride + r] = src[b * bh_stride + (int64_t)shift * D + r];
  }
}

}  // namespace kvr

using namespace kvr;

// ====================================================================== C ABI
extern "C" int kvr_pack_unsigned(const uint8_t* codes, int64_t n, int bits, uint8_t* payload,
                                 kvr_stream_t stream) {
  if (bits < 1 || bits > 8 || n < 0) return KVR_ERR_INVALID_ARGUMENT;
  if (n == 0) return KVR_OK;
  if (!codes || !payload) return KVR_ERR_INVALID_ARGUMENT;
  const int64_t nbytes = (n * bits + 7) / 8;
  pack_unsigned_kernel<<<grid_for(nbytes, 256), 256, 0, as_stream(stream)>>>(codes, n, bits, payload, nbytes);
  return check_launch();
}

extern "C" int kvr_unpack_unsigned(const uint8_t* payload, int64_t n, int bits, uint8_t* codes,
                                   kvr_stream_t stream) {
  if (bits < 1 || bits > 8 || n < 0) return KVR_ERR_INVALID_ARGUMENT;
  if (n == 0) return KVR_OK;
  if (!codes || !payload) return KVR_ERR_INVALID_ARGUMENT;
  const int64_t nbytes = (n * bits + 7) / 8;
  unpack_unsigned_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(payload, nbytes, n, bits, codes);
  return check_launch();
}

extern "C" int kvr_quantize_per_token(const kvr_token_quant_args* a, kvr_stream_t stream) {
  if (!a || a->bits < 2 || a->bits > 8 || a->head_dim <= 0 || a->head_dim > kMaxD || a->bh < 0 ||
      a->rows < 0 || a->row0 < 0)
    return KVR_ERR_INVALID_ARGUMENT;
  if (a->bh == 0 || a->rows == 0) return KVR_OK;
  if (!a->x || !a->payload || !a->scale || !a->offset) return KVR_ERR_INVALID_ARGUMENT;
  const bool generic = ((int64_t)a->head_dim * a->bits) % 8 != 0;
  // Generic path: the payload is the flat stream of [bh, rows, D] codes
  // (payload_bh_stride is not used).
  if (generic && (!a->codes_scratch || a->row0 != 0)) return KVR_ERR_INVALID_ARGUMENT;
  const int64_t total = (int64_t)a->bh * a->rows;
  quant_token_kernel<<<grid_for(total, kTokWarps), kTokWarps * 32, 0, as_stream(stream)>>>(*a, generic);
  int st = check_launch();
  if (st != KVR_OK || !generic) return st;
  return kvr_pack_unsigned(a->codes_scratch, total * a->head_dim, a->bits, a->payload, stream);
}

extern "C" int kvr_quantize_grouped(const kvr_group_quant_args* a, kvr_stream_t stream) {
  if (!a || a->bits < 2 || a->bits > 8 || a->head_dim <= 0 || a->head_dim > 1024 ||
      a->group_size <= 0 || a->bh < 0 || a->groups < 0 || a->group0 < 0)
    return KVR_ERR_INVALID_ARGUMENT;
  if (a->bh == 0 || a->groups == 0) return KVR_OK;
  if (!a->x || !a->payload || !a->scale || !a->offset) return KVR_ERR_INVALID_ARGUMENT;
  const bool generic = ((int64_t)a->head_dim * a->bits) % 8 != 0;
  const int64_t smem = generic ? 0 : (int64_t)a->group_size * a->head_dim;
  if (smem > 200 * 1024) return KVR_ERR_UNSUPPORTED;
  if (generic && (!a->codes_scratch || a->group0 != 0)) return KVR_ERR_INVALID_ARGUMENT;
  int threads = ((std::min(a->head_dim, 1024) + 31) / 32) * 32;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(quant_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  }
  const int64_t total = (int64_t)a->bh * a->groups;
  const int grid = (int)std::min<int64_t>(total, 148 * 16);
  quant_group_kernel<<<grid, threads, (size_t)smem, as_stream(stream)>>>(*a, generic);
  int st = check_launch();
  if (st != KVR_OK || !generic) return st;
  const int64_t n = (int64_t)a->bh * a->groups * a->group_size * a->head_dim;
  return kvr_pack_unsigned(a->codes_scratch, n, a->bits, a->payload, stream);
}

extern "C" int kvr_dequantize(const kvr_dequant_args* a, kvr_stream_t stream) {
  if (!a || a->bits < 1 || a->bits > 8 || a->head_dim <= 0 || a->bh < 0 || a->seq_len < 0 ||
      a->out_dtype < 0 || a->out_dtype > 2)
    return KVR_ERR_INVALID_ARGUMENT;
  const bool keys = a->group_size > 0;
  if (keys && (a->prefix_len < 0 || a->prefix_len > a->seq_len || a->prefix_len % a->group_size))
    return KVR_ERR_INVALID_ARGUMENT;
  if ((int64_t)a->bh * a->seq_len == 0) return KVR_OK;
  if (!a->out) return KVR_ERR_INVALID_ARGUMENT;
  const int P = keys ? a->prefix_len : a->seq_len;
  if (P > 0 && (!a->payload || !a->scale || !a->offset)) return KVR_ERR_INVALID_ARGUMENT;
  if (keys && P < a->seq_len && !a->residual) return KVR_ERR_INVALID_ARGUMENT;
  const int flat = ((int64_t)a->head_dim * a->bits) % 8 != 0;
  const int64_t total = (int64_t)a->bh * a->seq_len * a->head_dim;
  dequant_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(*a, flat);
  return check_launch();
}

extern "C" int kvr_append(const kvr_append_args* a, kvr_stream_t stream) {
  if (!a || a->head_dim <= 0 || a->head_dim > kMaxD || a->value_bits < 2 || a->value_bits > 8 ||
      a->bh < 0 || a->n < 0 || a->seq_len < 0 || a->res_len < 0)
    return KVR_ERR_INVALID_ARGUMENT;
  if (((int64_t)a->head_dim * a->value_bits) % 8 != 0) return KVR_ERR_UNSUPPORTED;
  if (a->res_len + a->n > a->res_capacity || a->seq_len + a->n > a->seq_capacity) return KVR_ERR_CAPACITY;
  if (a->bh == 0 || a->n == 0) return KVR_OK;
  if (!a->k || !a->v || !a->key_residual || !a->value_payload || !a->value_scale || !a->value_offset)
    return KVR_ERR_INVALID_ARGUMENT;
  const int64_t total = (int64_t)a->bh * a->n;
  append_kernel<<<grid_for(total, kTokWarps), kTokWarps * 32, 0, as_stream(stream)>>>(*a, nullptr);
  return check_launch();
}

// ------------------------------------------------ lengths in device memory
// lengths[0] = sequence length, lengths[1] = quantized prefix length,
// lengths[2] = error flag (non-zero after an append past a capacity).
__global__ void set_lengths_kernel(int* lengths, int seq_len, int prefix_len) {
  lengths[0] = seq_len;
  lengths[1] = prefix_len;
}
__global__ void advance_lengths_kernel(int* lengths, int n) {
  if (lengths[2] == 0) lengths[0] += n;
}

extern "C" int kvr_append_lengths(const kvr_append_args* a, int* lengths, kvr_stream_t stream) {
  if (!a || !lengths || a->head_dim <= 0 || a->head_dim > kMaxD || a->value_bits < 2 || a->value_bits > 8 ||
      a->bh < 0 || a->n < 0 || a->res_capacity < 0 || a->seq_capacity < 0)
    return KVR_ERR_INVALID_ARGUMENT;
  if (((int64_t)a->head_dim * a->value_bits) % 8 != 0) return KVR_ERR_UNSUPPORTED;
  if (a->bh == 0 || a->n == 0) return KVR_OK;
  if (!a->k || !a->v || !a->key_residual || !a->value_payload || !a->value_scale || !a->value_offset)
    return KVR_ERR_INVALID_ARGUMENT;
  const int64_t total = (int64_t)a->bh * a->n;
  append_kernel<<<grid_for(total, kTokWarps), kTokWarps * 32, 0, as_stream(stream)>>>(*a, lengths);
  return check_launch();
}

extern "C" int kvr_set_lengths(int* lengths, int seq_len, int prefix_len, kvr_stream_t stream) {
  if (!lengths || seq_len < 0 || prefix_len < 0 || prefix_len > seq_len) return KVR_ERR_INVALID_ARGUMENT;
  set_lengths_kernel<<<1, 1, 0, as_stream(stream)>>>(lengths, seq_len, prefix_len);
  return check_launch();
}

extern "C" int kvr_advance_lengths(int* lengths, int n, kvr_stream_t stream) {
  if (!lengths || n < 0) return KVR_ERR_INVALID_ARGUMENT;
  advance_lengths_kernel<<<1, 1, 0, as_stream(stream)>>>(lengths, n);
  return check_launch();
}

extern "C" int kvr_flush_groups(const kvr_flush_args* a, kvr_stream_t stream) {
  if (!a || a->groups < 0 || a->group_size <= 0 || a->res_len < 0 || a->prefix_len < 0 ||
      a->prefix_len % a->group_size || a->groups * a->group_size > a->res_len)
    return KVR_ERR_INVALID_ARGUMENT;
  if (a->prefix_len + a->groups * a->group_size > a->prefix_capacity) return KVR_ERR_CAPACITY;
  if (((int64_t)a->head_dim * a->key_bits) % 8 != 0) return KVR_ERR_UNSUPPORTED;
  if (a->bh == 0) return KVR_OK;
  if (a->residual_in == a->residual_out) return KVR_ERR_INVALID_ARGUMENT;
  if (a->groups > 0) {
    kvr_group_quant_args q{};
    q.x = a->residual_in; q.x_bh_stride = a->residual_bh_stride; q.x_row_stride = a->head_dim;
    q.payload = a->key_payload; q.payload_bh_stride = a->key_payload_bh_stride;
    q.scale = a->key_scale; q.offset = a->key_offset; q.meta_bh_stride = a->key_meta_bh_stride;
    q.bh = a->bh; q.groups = a->groups; q.group0 = a->prefix_len / a->group_size;
    q.group_size = a->group_size; q.head_dim = a->head_dim; q.bits = a->key_bits;
    q.codes_scratch = nullptr;
    int st = kvr_quantize_grouped(&q, stream);
    if (st != KVR_OK) return st;
  }
  const int shift = a->groups * a->group_size;
  const int keep = a->res_len - shift;
  if (keep > 0) {
    const int64_t total = (int64_t)a->bh * keep * a->head_dim;
    residual_move_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
        a->residual_in, a->residual_out, a->residual_bh_stride, a->bh, shift, keep, a->head_dim);
    return check_launch();
  }
  return KVR_OK;
}
