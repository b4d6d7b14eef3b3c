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

// ============================================== fast paths (2/4/8-bit codes)
// Used when every packed row is whole bytes and the buffers are aligned for
// vector accesses; the kernels above remain for everything else.  Same
// arithmetic as the generic kernels, bit for bit.

// Per-token values, 8 lanes per row: lane l serves row (l >> 3) of a 4-row
// block and owns channels [(l & 7) * KL, +KL), KL = D / 8, loaded with
// 16-byte loads; the row's min/max takes three shuffles within its 8 lanes,
// and each lane stores its KL codes as one contiguous KL*BITS/8-byte piece.
// BPW blocks per warp iteration keep several rows' loads in flight.  Same
// arithmetic as the reference's per-row rule (exact min/max, IEEE scale,
// affine_code_rcp), so the codes and metadata are bit-identical to it.
template <int KL, int BITS, int BPW>
__global__ void __launch_bounds__(256) quant_token_fast(kvr_token_quant_args a) {
  constexpr int LB = KL * BITS / 8;   // packed bytes per lane
  constexpr int NW = (LB + 3) / 4;    // ... as 32-bit words
  constexpr int levels = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31, sub = lane & 7, rsel = lane >> 3;
  const int warp0 = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int nwarps = (int)((gridDim.x * blockDim.x) >> 5);
  constexpr int RB = 4 * BPW;                 // rows per warp iteration
  const int bpb = (a.rows + RB - 1) / RB;     // row blocks per b*h slab
  const int nblocks = a.bh * bpb;
  const int row_bytes = 8 * LB;
  for (int ib = warp0; ib < nblocks; ib += nwarps) {
    const int bh = ib / bpb;
    const int rb = (ib - bh * bpb) * RB;
    float xv[BPW][KL];
    bool ok[BPW];
#pragma unroll
    for (int u = 0; u < BPW; ++u) {
      const int r = rb + 4 * u + rsel;
      ok[u] = r < a.rows;
      if (ok[u]) {
        const uint16_t* x = a.x + (int64_t)bh * a.x_bh_stride + (int64_t)r * a.x_row_stride + sub * KL;
#pragma unroll
        for (int v = 0; v < KL / 8; ++v) {
          float t[8];
          load_bf16x<8>(x + 8 * v, t);
#pragma unroll
          for (int k = 0; k < 8; ++k) xv[u][8 * v + k] = t[k];
        }
      } else {
#pragma unroll
        for (int k = 0; k < KL; ++k) xv[u][k] = 0.f;   // keeps the group's shuffles defined
      }
    }
#pragma unroll
    for (int u = 0; u < BPW; ++u) {
      float mn = xv[u][0], mx = xv[u][0];
#pragma unroll
      for (int k = 1; k < KL; ++k) {
        mn = fminf(mn, xv[u][k]);
        mx = fmaxf(mx, xv[u][k]);
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) {   // within the row's 8 lanes
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      const float scale = affine_scale(mn, mx, BITS);
      const float inv = __frcp_rn(scale);
      uint32_t w[NW];
#pragma unroll
      for (int i = 0; i < NW; ++i) w[i] = 0u;
#pragma unroll
      for (int k = 0; k < KL; ++k)
        w[(k * BITS) / 32] |= affine_code_rcp(xv[u][k], mn, scale, inv, levels) << ((k * BITS) % 32);
      if (!ok[u]) continue;
      const int r = rb + 4 * u + rsel;
      uint8_t* dst = a.payload + (int64_t)bh * a.payload_bh_stride + (int64_t)(a.row0 + r) * row_bytes + sub * LB;
      if constexpr (LB == 2) {
        *reinterpret_cast<uint16_t*>(dst) = (uint16_t)w[0];
      } else if constexpr (LB == 4) {
        *reinterpret_cast<uint32_t*>(dst) = w[0];
      } else if constexpr (LB == 8) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
      } else {
#pragma unroll
        for (int i = 0; i < LB / 16; ++i)
          reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
      if (sub == 0) {
        const int64_t m = (int64_t)bh * a.meta_bh_stride + a.row0 + r;
        a.scale[m] = f32_to_bf16_bits(scale);
        a.offset[m] = f32_to_bf16_bits(mn);
      }
    }
  }
}

// Grouped keys (G <= 32): a thread per (b*h, group, channel quad); a first
// pass over the group's G rows takes the per-channel min/max (one 8-byte
// load per row; a warp reads 32 consecutive quads of a row), the second
// re-reads them (L1) to emit the codes, one store of the packed quad per row.
template <int G, int BITS>
__global__ void __launch_bounds__(256) quant_group_fast(kvr_group_quant_args a) {
  constexpr int QB = 4 * BITS / 8;   // packed bytes per quad
  constexpr int levels = (1 << BITS) - 1;
  const int D = a.head_dim, Q = D / 4;
  const int row_bytes = D * BITS / 8;
  const int total = a.bh * a.groups * Q;
  for (int tid = blockIdx.x * blockDim.x + threadIdx.x; tid < total; tid += gridDim.x * blockDim.x) {
    const int item = tid / Q;
    const int j = tid - item * Q;
    const int bh = item / a.groups;
    const int gi = item - bh * a.groups;
    const int g = a.group0 + gi;
    const uint16_t* x = a.x + (int64_t)bh * a.x_bh_stride + (int64_t)gi * G * a.x_row_stride + 4 * j;
    float mn[4], mx[4];
    {
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(x));
      mn[0] = mx[0] = bf16lo(w.x); mn[1] = mx[1] = bf16hi(w.x);
      mn[2] = mx[2] = bf16lo(w.y); mn[3] = mx[3] = bf16hi(w.y);
    }
#pragma unroll 8
    for (int t = 1; t < G; ++t) {
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(x + (int64_t)t * a.x_row_stride));
      const float v[4] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y)};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        mn[c] = fminf(mn[c], v[c]);
        mx[c] = fmaxf(mx[c], v[c]);
      }
    }
    float sc[4], inv[4];
    uint32_t sbits[2] = {0u, 0u}, zbits[2] = {0u, 0u};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      sc[c] = affine_scale(mn[c], mx[c], BITS);
      inv[c] = __frcp_rn(sc[c]);
      sbits[c >> 1] |= (uint32_t)f32_to_bf16_bits(sc[c]) << (16 * (c & 1));
      zbits[c >> 1] |= (uint32_t)f32_to_bf16_bits(mn[c]) << (16 * (c & 1));
    }
    const int64_t meta = (int64_t)bh * a.meta_bh_stride + (int64_t)g * D + 4 * j;
    *reinterpret_cast<uint2*>(a.scale + meta) = make_uint2(sbits[0], sbits[1]);
    *reinterpret_cast<uint2*>(a.offset + meta) = make_uint2(zbits[0], zbits[1]);
    uint8_t* dst = a.payload + (int64_t)bh * a.payload_bh_stride + (int64_t)g * G * row_bytes + j * QB;
#pragma unroll 8
    for (int t = 0; t < G; ++t) {
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(x + (int64_t)t * a.x_row_stride));
      const float v[4] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y)};
      uint32_t word = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) word |= affine_code_rcp(v[c], mn[c], sc[c], inv[c], levels) << (c * BITS);
      store_bytes<QB>(dst + (int64_t)t * row_bytes, word);
    }
  }
}

// Dequantize: a thread per 8 consecutive outputs of a row (codes of the
// 8 channels are BITS bytes; key metadata for them one 16-byte load each).
template <int BITS, int OUT>
__global__ void __launch_bounds__(256) dequant_fast(kvr_dequant_args a) {
  const int D = a.head_dim, S = a.seq_len, C8 = D / 8;
  const bool keys = a.group_size > 0;
  const int P = keys ? a.prefix_len : S;
  const int64_t row_bytes = (int64_t)D * BITS / 8;
  const int total = a.bh * S * C8;   // < 2^31 (checked by the launcher)
  for (int tid = blockIdx.x * blockDim.x + threadIdx.x; tid < total; tid += gridDim.x * blockDim.x) {
    const int row = tid / C8;
    const int c = tid - row * C8;
    const int bh = row / S;
    const int t = row - bh * S;
    float v[8];
    if (t < P) {
      const uint8_t* src = a.payload + (int64_t)bh * a.payload_bh_stride + (int64_t)t * row_bytes + (int64_t)c * BITS;
      uint64_t w;
      if constexpr (BITS == 2) w = *reinterpret_cast<const uint16_t*>(src);
      else if constexpr (BITS == 4) w = *reinterpret_cast<const uint32_t*>(src);
      else {
        const uint2 x = *reinterpret_cast<const uint2*>(src);
        w = (uint64_t)x.x | ((uint64_t)x.y << 32);
      }
      if (keys) {
        const int64_t meta = (int64_t)bh * a.meta_bh_stride + (int64_t)(t / a.group_size) * D + 8 * c;
        float s[8], z[8];
        load_bf16x<8>(a.scale + meta, s);
        load_bf16x<8>(a.offset + meta, z);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = affine_dequant((uint32_t)(w >> (i * BITS)) & ((1u << BITS) - 1u), s[i], z[i]);
      } else {
        const int64_t meta = (int64_t)bh * a.meta_bh_stride + t;
        const float s = bf16_bits_to_f32(a.scale[meta]), z = bf16_bits_to_f32(a.offset[meta]);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = affine_dequant((uint32_t)(w >> (i * BITS)) & ((1u << BITS) - 1u), s, z);
      }
    } else {
      load_bf16x<8>(a.residual + (int64_t)bh * a.residual_bh_stride + (int64_t)(t - P) * D + 8 * c, v);
    }
    const int64_t o = (int64_t)row * D + 8 * c;
    if constexpr (OUT == 1) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + o);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (OUT == 2) {
          const __half2 x = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
          h[i] = *reinterpret_cast<const uint32_t*>(&x);
        } else {
          h[i] = (uint32_t)f32_to_bf16_bits(v[2 * i]) | ((uint32_t)f32_to_bf16_bits(v[2 * i + 1]) << 16);
        }
      }
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + o) = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
}

// pack_unsigned / unpack_unsigned, 16 codes per thread; the last partial
// group of 16 is handled byte by byte.
template <int BITS>
__global__ void pack_unsigned_fast(const uint8_t* __restrict__ codes, int64_t n, uint8_t* __restrict__ payload) {
  constexpr uint32_t mask = (1u << BITS) - 1u;
  const int64_t n16 = n / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n16; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n16) {
      const uint4 c = reinterpret_cast<const uint4*>(codes)[i];
      if constexpr (BITS == 8) {
        reinterpret_cast<uint4*>(payload)[i] = c;   // 8-bit codes are their own stream
      } else {
        const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
        uint64_t w = 0;
#pragma unroll
        for (int k = 0; k < 16; ++k) w |= (uint64_t)((cw[k >> 2] >> (8 * (k & 3))) & mask) << (k * BITS);
        store_bytes<2 * BITS>(payload + i * (2 * BITS), w);
      }
    } else {
      const int64_t b0 = n16 * 2 * BITS, nbytes = (n * BITS + 7) / 8;
      for (int64_t b = b0; b < nbytes; ++b)
        payload[b] = (uint8_t)stream_byte(b, BITS, n, [&](int64_t j) { return (uint32_t)codes[j]; });
    }
  }
}

template <int BITS>
__global__ void unpack_unsigned_fast(const uint8_t* __restrict__ payload, int64_t n, uint8_t* __restrict__ codes) {
  constexpr uint32_t mask = (1u << BITS) - 1u;
  const int64_t n16 = n / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n16; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n16) {
      const uint8_t* src = payload + i * (2 * BITS);
      uint64_t w;
      if constexpr (BITS == 2) w = *reinterpret_cast<const uint32_t*>(src);
      else if constexpr (BITS == 4) {
        const uint2 x = *reinterpret_cast<const uint2*>(src);
        w = (uint64_t)x.x | ((uint64_t)x.y << 32);
      } else {
        w = 0;   // 8-bit codes are the payload itself
      }
      uint32_t out[4];
      if constexpr (BITS == 8) {
        const uint4 x = *reinterpret_cast<const uint4*>(src);
        out[0] = x.x; out[1] = x.y; out[2] = x.z; out[3] = x.w;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) o |= (uint32_t)((w >> ((4 * q + k) * BITS)) & mask) << (8 * k);
          out[q] = o;
        }
      }
      reinterpret_cast<uint4*>(codes)[i] = make_uint4(out[0], out[1], out[2], out[3]);
    } else {
      for (int64_t j = n16 * 16; j < n; ++j) {
        const int64_t bit = j * BITS;
        codes[j] = (uint8_t)((payload[bit >> 3] >> (bit & 7)) & mask);
      }
    }
  }
}

static inline bool al(const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// ============================================================ streaming cache
// Append: warp per (bh, new token).  Key row copied into the BF16 residual
// window; value row quantized per token at row seq_len + i.
// After an append from device-side lengths: the last block to finish moves
// the sequence length on by n (lengths[3] counts finished blocks, left zero).
__device__ __forceinline__ void advance_after_append(int* lengths, int n) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(lengths + 3, 1) == (int)gridDim.x - 1) {
      lengths[3] = 0;
      lengths[0] += n;
    }
  }
}

__global__ void __launch_bounds__(kTokWarps * 32) append_kernel(kvr_append_args a, int* lengths, int advance) {
  __shared__ uint8_t codes_s[kTokWarps][kMaxD];
  pdl_enter();
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
  if (lengths && advance) advance_after_append(lengths, a.n);
}

// Append, vectorised (D in {64,128,256}, 2/4/8-bit values): a warp per new
// token row; lane l copies key channels [l*K, l*K+K) and quantizes the same
// value channels in registers (min/max by warp shuffles, the per-token rule).
template <int K, int BITS>
__global__ void __launch_bounds__(256) append_fast(kvr_append_args a, int* lengths, int advance) {
  pdl_enter();
  constexpr int LB = K * BITS / 8;
  constexpr int levels = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31;
  if (lengths) {
    const int S = *reinterpret_cast<volatile int*>(lengths);
    const int P = *reinterpret_cast<volatile int*>(lengths + 1);
    if (P < 0 || P > S || S + a.n > a.seq_capacity || S - P + a.n > a.res_capacity) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(lengths + 2, 1);
      return;
    }
    a.seq_len = S;
    a.res_len = S - P;
  }
  const int total = a.bh * a.n;
  const int nwarps = (int)((gridDim.x * blockDim.x) >> 5);
  for (int item = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); item < total; item += nwarps) {
    const int bh = item / a.n;
    const int i = item - bh * a.n;
    const int64_t src = (int64_t)item * (32 * K) + lane * K;
    // key row -> BF16 residual window (K bf16 per lane)
    uint16_t* kr = a.key_residual + (int64_t)bh * a.key_residual_bh_stride + (int64_t)(a.res_len + i) * (32 * K) +
                   lane * K;
    if constexpr (K == 2) *reinterpret_cast<uint32_t*>(kr) = *reinterpret_cast<const uint32_t*>(a.k + src);
    else if constexpr (K == 4) *reinterpret_cast<uint2*>(kr) = *reinterpret_cast<const uint2*>(a.k + src);
    else *reinterpret_cast<uint4*>(kr) = *reinterpret_cast<const uint4*>(a.k + src);
    float xv[K];
    load_bf16x<K>(a.v + src, xv);
    float mn = xv[0], mx = xv[0];
#pragma unroll
    for (int k = 1; k < K; ++k) {
      mn = fminf(mn, xv[k]);
      mx = fmaxf(mx, xv[k]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = affine_scale(mn, mx, BITS);
    const float inv = __frcp_rn(scale);
    uint64_t w = 0;
#pragma unroll
    for (int k = 0; k < K; ++k) w |= (uint64_t)affine_code_rcp(xv[k], mn, scale, inv, levels) << (k * BITS);
    store_bytes<LB>(a.value_payload + (int64_t)bh * a.value_payload_bh_stride + (int64_t)(a.seq_len + i) * (32 * LB) +
                        lane * LB, w);
    if (lane == 0) {
      const int64_t meta = (int64_t)bh * a.value_meta_bh_stride + a.seq_len + i;
      a.value_scale[meta] = f32_to_bf16_bits(scale);
      a.value_offset[meta] = f32_to_bf16_bits(mn);
    }
  }
  if (lengths && advance) advance_after_append(lengths, a.n);
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

// Append launcher: the vectorised kernel where the layout allows it.
static int launch_append(const kvr_append_args* a, int* lengths, int advance, cudaStream_t s) {
  const int64_t total = (int64_t)a->bh * a->n;
  const int D = a->head_dim, bits = a->value_bits, K = D / 32;
  const bool fast = total < (1ll << 30) && (D == 64 || D == 128 || D == 256) && (bits == 2 || bits == 4 || bits == 8) &&
                    (K * bits) % 8 == 0 && al(a->k, 16) && al(a->v, 16) && al(a->key_residual, 16) &&
                    a->key_residual_bh_stride % 8 == 0 && al(a->value_payload, 16) &&
                    a->value_payload_bh_stride % 8 == 0;
  if (fast) {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 7) / 8, 148 * 64));
#define KVR_APP(K_, B_) \
  if (K == K_ && bits == B_) (void)pdl_launch(append_fast<K_, B_>, dim3(grid), dim3(256), 0, s, 1, *a, lengths, advance);
    KVR_APP(2, 4) KVR_APP(2, 8) KVR_APP(4, 2) KVR_APP(4, 4) KVR_APP(4, 8) KVR_APP(8, 2) KVR_APP(8, 4) KVR_APP(8, 8)
#undef KVR_APP
    return check_launch();
  }
  (void)pdl_launch(append_kernel, dim3(grid_for(total, kTokWarps)), dim3(kTokWarps * 32), 0, s, 1, *a, lengths,
                   advance);
  return check_launch();
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
  if ((bits == 2 || bits == 4 || bits == 8) && al(codes, 16) && al(payload, 16)) {
    const int grid = grid_for(n / 16 + 1, 256);
    if (bits == 2) pack_unsigned_fast<2><<<grid, 256, 0, as_stream(stream)>>>(codes, n, payload);
    else if (bits == 4) pack_unsigned_fast<4><<<grid, 256, 0, as_stream(stream)>>>(codes, n, payload);
    else pack_unsigned_fast<8><<<grid, 256, 0, as_stream(stream)>>>(codes, n, payload);
    return check_launch();
  }
  pack_unsigned_kernel<<<grid_for(nbytes, 256), 256, 0, as_stream(stream)>>>(codes, n, bits, payload, nbytes);
  return check_launch();
}

extern "C" int kvr_unpack_unsigned(const uint8_t* payload, int64_t n, int bits, uint8_t* codes,
                                   kvr_stream_t stream) {
  if (bits < 1 || bits > 8 || n < 0) return KVR_ERR_INVALID_ARGUMENT;
  if (n == 0) return KVR_OK;
  if (!codes || !payload) return KVR_ERR_INVALID_ARGUMENT;
  const int64_t nbytes = (n * bits + 7) / 8;
  if ((bits == 2 || bits == 4 || bits == 8) && al(codes, 16) && al(payload, 16)) {
    const int grid = grid_for(n / 16 + 1, 256);
    if (bits == 2) unpack_unsigned_fast<2><<<grid, 256, 0, as_stream(stream)>>>(payload, n, codes);
    else if (bits == 4) unpack_unsigned_fast<4><<<grid, 256, 0, as_stream(stream)>>>(payload, n, codes);
    else unpack_unsigned_fast<8><<<grid, 256, 0, as_stream(stream)>>>(payload, n, codes);
    return check_launch();
  }
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
  {
    const int D = a->head_dim, bits = a->bits, KL = D / 8;
    const bool fast = !generic && total < (1ll << 30) && (bits == 2 || bits == 4 || bits == 8) &&
                      (D == 64 || D == 128 || D == 256) && al(a->x, 16) && a->x_bh_stride % 8 == 0 &&
                      a->x_row_stride % 8 == 0 && al(a->payload, 16) && a->payload_bh_stride % 16 == 0;
    if (fast) {
      // warps of 4 rows per block: 2 blocks per iteration, 1 at D=256 (registers)
      const int bpw = KL == 32 ? 1 : 2;
      const int64_t warps = (total + 4 * bpw - 1) / (4 * bpw);
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, 148 * 64));
#define KVR_TOK(K_, B_, P_) \
  if (KL == K_ && bits == B_) quant_token_fast<K_, B_, P_><<<grid, 256, 0, as_stream(stream)>>>(*a);
      KVR_TOK(8, 2, 2) KVR_TOK(8, 4, 2) KVR_TOK(8, 8, 2) KVR_TOK(16, 2, 2) KVR_TOK(16, 4, 2) KVR_TOK(16, 8, 2)
      KVR_TOK(32, 2, 1) KVR_TOK(32, 4, 1) KVR_TOK(32, 8, 1)
#undef KVR_TOK
      return check_launch();
    }
  }
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
  {
    const int D = a->head_dim, G = a->group_size, bits = a->bits;
    const bool fast = !generic && total * (D / 4) < (1ll << 30) && (bits == 2 || bits == 4 || bits == 8) &&
                      D % 4 == 0 &&
                      (G == 16 || G == 32) && al(a->x, 8) && a->x_bh_stride % 4 == 0 &&
                      a->x_row_stride % 4 == 0 && al(a->payload, 4) && a->payload_bh_stride % 4 == 0 &&
                      al(a->scale, 8) && al(a->offset, 8) && a->meta_bh_stride % 4 == 0;
    if (fast) {
      const int64_t threads_total = total * (D / 4);
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((threads_total + 255) / 256, 148 * 64));
#define KVR_GRP(G_, B_) \
  if (G == G_ && bits == B_) quant_group_fast<G_, B_><<<grid, 256, 0, as_stream(stream)>>>(*a);
      KVR_GRP(16, 2) KVR_GRP(16, 4) KVR_GRP(16, 8) KVR_GRP(32, 2) KVR_GRP(32, 4) KVR_GRP(32, 8)
#undef KVR_GRP
      return check_launch();
    }
  }
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
  const int bits = a->bits, od = a->out_dtype;
  const bool fast = !flat && total / 8 < (1ll << 30) && (bits == 2 || bits == 4 || bits == 8) &&
                    a->head_dim % 8 == 0 && al(a->out, 16) &&
                    (P == 0 || (al(a->payload, 8) && a->payload_bh_stride % 8 == 0)) &&
                    (P == 0 || !keys || (al(a->scale, 16) && al(a->offset, 16) && a->meta_bh_stride % 8 == 0)) &&
                    (P == a->seq_len || (al(a->residual, 16) && a->residual_bh_stride % 8 == 0));
  if (fast) {
    const int grid = grid_for(total / 8, 256);
#define KVR_DQ(B_, O_) \
  if (bits == B_ && od == O_) dequant_fast<B_, O_><<<grid, 256, 0, as_stream(stream)>>>(*a);
    KVR_DQ(2, 0) KVR_DQ(2, 1) KVR_DQ(2, 2) KVR_DQ(4, 0) KVR_DQ(4, 1) KVR_DQ(4, 2) KVR_DQ(8, 0) KVR_DQ(8, 1)
    KVR_DQ(8, 2)
#undef KVR_DQ
    return check_launch();
  }
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
  return launch_append(a, nullptr, 0, as_stream(stream));
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

extern "C" int kvr_append_lengths(const kvr_append_args* a, int* lengths, int advance, kvr_stream_t stream) {
  if (!a || !lengths || a->head_dim <= 0 || a->head_dim > kMaxD || a->value_bits < 2 || a->value_bits > 8 ||
      a->bh < 0 || a->n < 0 || a->res_capacity < 0 || a->seq_capacity < 0)
    return KVR_ERR_INVALID_ARGUMENT;
  if (((int64_t)a->head_dim * a->value_bits) % 8 != 0) return KVR_ERR_UNSUPPORTED;
  if (a->bh == 0 || a->n == 0) return KVR_OK;
  if (!a->k || !a->v || !a->key_residual || !a->value_payload || !a->value_scale || !a->value_offset)
    return KVR_ERR_INVALID_ARGUMENT;
  return launch_append(a, lengths, advance, as_stream(stream));
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
