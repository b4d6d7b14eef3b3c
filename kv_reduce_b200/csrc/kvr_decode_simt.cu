// Packed-KV decode attention on the CUDA cores (fp32 FMA, no tensor cores),
// sm_100a.  The measured A/B baseline for the tensor-core kernel in
// kvr_decode.cu: same packed layout, same inputs and outputs, same split-K +
// LSE-merge structure, with the GQA group's query heads sharing every packed
// byte as there.  Reference computation: triton_packed_kv_attention.py:134-281
// (dequantize q*scale+offset in fp32, scores q.k/sqrt(D), online softmax,
// values dequantized per token, LSE merge of the splits).
//
// Per CTA (4 warps): one (layer, b, kv head, split).  Per warp, 32-token
// chunks of one key group:
//   * the group-scaled query q~[d][h] = q[h][d] * s[d] (fp32) and the bias
//     q.z per head go to the warp's shared memory (lane = channel);
//   * scores: lane = token, fp32 FMA of the key codes against q~ (broadcast
//     shared-memory reads, all heads of a channel in one 16/32-byte load);
//     BF16 residual rows against the raw query;
//   * online softmax per head across the warp (shuffles, exp2);
//   * P V: lane = D/32 contiguous channels, token by token: codes
//     dequantized as c * s_t + z_t (fp32) and accumulated into every head.
// The warps merge in shared memory; the split partials (m, l, o) go to the
// workspace and a second kernel merges them into the output.
#include "kvr_common.cuh"

#include <algorithm>
#include <cmath>

namespace kvr {
namespace simt {

constexpr int kWarps = 4;
constexpr int kChunk = 32;

struct Layer {
  const uint8_t* kp;
  const uint16_t* ks;
  const uint16_t* ko;
  const uint16_t* kr;
  const uint8_t* vp;
  const uint16_t* vs;
  const uint16_t* vo;
  const uint16_t* q;
  void* out;
};

struct Args {
  Layer L[KVR_MAX_LAYERS];
  int BH, HKV, HQ, S, P, log2G, ns, cps, out_f32;
  int64_t kp_bh, km_bh, kr_bh, vp_bh, vm_bh;
  float cs;       // log2(e) / sqrt(D)
  float* part;    // [items][GQA][2 + D]: m, l, o
};

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int D, int KB, int VB, int GQA>
struct SCfg {
  static constexpr int HP = (GQA + 3) / 4 * 4;       // heads padded to a 16-byte row of floats
  static constexpr int CPL = D / 32;                 // P V channels per lane
  static constexpr int RBK = D * KB / 8;             // key payload bytes per token
  static constexpr int RBV = D * VB / 8;
  static constexpr int QF_OFF = 0;                                   // [D][HP] raw query
  static constexpr int QT_OFF = QF_OFF + D * HP * 4;                 // [warp][D][HP] scaled query
  static constexpr int PW_OFF = QT_OFF + kWarps * D * HP * 4;        // [warp][32][HP] probabilities
  static constexpr int SMEM = PW_OFF + kWarps * kChunk * HP * 4;
  static_assert(D % 32 == 0 && (D * KB) % 128 == 0, "key rows of whole 16-byte pieces");
  static_assert((CPL * VB) % 8 == 0, "a lane's value bits fill whole bytes");
};

template <int D, int KB, int VB, int GQA>
__global__ void __launch_bounds__(kWarps * 32, 4) partial_kernel(const __grid_constant__ Args a) {
  using C = SCfg<D, KB, VB, GQA>;
  constexpr int HP = C::HP;
  extern __shared__ __align__(16) uint8_t smem[];
  float* qf = reinterpret_cast<float*>(smem + C::QF_OFF);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* qt = reinterpret_cast<float*>(smem + C::QT_OFF) + warp * D * HP;
  float* pw = reinterpret_cast<float*>(smem + C::PW_OFF) + warp * kChunk * HP;
  const float NEG_INF = -__int_as_float(0x7f800000);

  const int item = blockIdx.x;
  const int sp = item % a.ns, unit = item / a.ns;
  const int bh = unit % a.BH, layer = unit / a.BH;
  const int b = bh / a.HKV, kvh = bh % a.HKV;
  const Layer& Lp = a.L[layer];
  const uint8_t* kp = Lp.kp + (int64_t)bh * a.kp_bh;
  const uint16_t* ksc = Lp.ks + (int64_t)bh * a.km_bh;
  const uint16_t* kof = Lp.ko + (int64_t)bh * a.km_bh;
  const uint16_t* kres = Lp.kr + (int64_t)bh * a.kr_bh;
  const uint8_t* vp = Lp.vp + (int64_t)bh * a.vp_bh;
  const uint16_t* vsc = Lp.vs + (int64_t)bh * a.vm_bh;
  const uint16_t* vof = Lp.vo + (int64_t)bh * a.vm_bh;
  const uint16_t* q = Lp.q + ((int64_t)b * a.HQ + kvh * GQA) * D;

  for (int i = threadIdx.x; i < D * HP; i += blockDim.x) {
    const int d = i / HP, h = i % HP;
    qf[i] = h < GQA ? bf16_bits_to_f32(q[h * D + d]) : 0.f;
  }
  __syncthreads();

  float m[GQA], l[GQA], o[GQA][C::CPL];
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    m[h] = NEG_INF;
    l[h] = 0.f;
#pragma unroll
    for (int j = 0; j < C::CPL; ++j) o[h][j] = 0.f;
  }

  const int nch = (a.S + kChunk - 1) / kChunk;
  const int c0 = sp * a.cps, c1 = min(nch, c0 + a.cps);
  for (int c = c0 + warp; c < c1; c += kWarps) {
    const int tok0 = c * kChunk;
    const int t = tok0 + lane;
    const bool valid = t < a.S;
    float sc[GQA];
    if (tok0 < a.P) {   // a whole chunk of one key group (P and G are multiples of 32)
      const int grp = tok0 >> a.log2G;
      float bias[GQA];
#pragma unroll
      for (int h = 0; h < GQA; ++h) bias[h] = 0.f;
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        const int d = lane + 32 * j;
        const float s = bf16_bits_to_f32(ksc[(int64_t)grp * D + d]);
        const float z = bf16_bits_to_f32(kof[(int64_t)grp * D + d]);
#pragma unroll
        for (int h = 0; h < GQA; ++h) {
          const float qv = qf[d * HP + h];
          qt[d * HP + h] = qv * s;
          bias[h] = fmaf(qv, z, bias[h]);
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) bias[h] = warp_sum(bias[h]);
      __syncwarp();
      float acc[GQA];
#pragma unroll
      for (int h = 0; h < GQA; ++h) acc[h] = 0.f;
      if (valid) {
        const uint4* row = reinterpret_cast<const uint4*>(kp + (int64_t)t * C::RBK);
#pragma unroll
        for (int v = 0; v < C::RBK / 16; ++v) {
          const uint4 x = __ldg(row + v);
          const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
            for (int e = 0; e < 32 / KB; ++e) {
              const int d = (v * 4 + wi) * (32 / KB) + e;   // LSB-first codes
              const float cf = (float)((w4[wi] >> (KB * e)) & ((1u << KB) - 1u));
              const float* qd = qt + d * HP;
#pragma unroll
              for (int h = 0; h < GQA; ++h) acc[h] = fmaf(qd[h], cf, acc[h]);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) sc[h] = valid ? (acc[h] + bias[h]) * a.cs : NEG_INF;
    } else {            // BF16 residual rows
      float acc[GQA];
#pragma unroll
      for (int h = 0; h < GQA; ++h) acc[h] = 0.f;
      if (valid) {
        const uint4* row = reinterpret_cast<const uint4*>(kres + (int64_t)(t - a.P) * D);
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
          const uint4 x = __ldg(row + v);
          const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const int d = v * 8 + wi * 2;
            const float k0 = bf16lo(w4[wi]), k1 = bf16hi(w4[wi]);
#pragma unroll
            for (int h = 0; h < GQA; ++h) acc[h] = fmaf(qf[(d + 1) * HP + h], k1, fmaf(qf[d * HP + h], k0, acc[h]));
          }
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) sc[h] = valid ? acc[h] * a.cs : NEG_INF;
    }

    // online softmax per head over the chunk's tokens
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      const float mn = fmaxf(m[h], warp_max(sc[h]));
      const float alpha = (mn == NEG_INF) ? 1.f : exp2f(m[h] - mn);
      const float p = (mn == NEG_INF) ? 0.f : exp2f(sc[h] - mn);
      l[h] = fmaf(l[h], alpha, warp_sum(p));
      m[h] = mn;
#pragma unroll
      for (int j = 0; j < C::CPL; ++j) o[h][j] *= alpha;
      pw[lane * HP + h] = p;
    }
    // value scale / offset of the lane's token, shared by shuffles
    const float vs_l = valid ? bf16_bits_to_f32(vsc[t]) : 0.f;
    const float vz_l = valid ? bf16_bits_to_f32(vof[t]) : 0.f;
    __syncwarp();

    // P V: lane = channels [lane*CPL, +CPL)
    const int n_tok = min(kChunk, a.S - tok0);
    for (int tt = 0; tt < n_tok; ++tt) {
      const float s_t = __shfl_sync(0xffffffffu, vs_l, tt);
      const float z_t = __shfl_sync(0xffffffffu, vz_l, tt);
      const uint8_t* vrow = vp + (int64_t)(tok0 + tt) * C::RBV + lane * (C::CPL * VB / 8);
      uint32_t bits;
      if constexpr (C::CPL * VB / 8 == 4) bits = __ldg(reinterpret_cast<const uint32_t*>(vrow));
      else if constexpr (C::CPL * VB / 8 == 2) bits = __ldg(reinterpret_cast<const uint16_t*>(vrow));
      else bits = __ldg(vrow);
      const float* pt = pw + tt * HP;
#pragma unroll
      for (int j = 0; j < C::CPL; ++j) {
        const float v = fmaf((float)((bits >> (VB * j)) & ((1u << VB) - 1u)), s_t, z_t);
#pragma unroll
        for (int h = 0; h < GQA; ++h) o[h][j] = fmaf(pt[h], v, o[h][j]);
      }
    }
    __syncwarp();
  }

  // merge the warps (shared memory reused), then store this split's partial
  __syncthreads();
  float* mo = reinterpret_cast<float*>(smem);                 // [warp][GQA][D]
  float* mm = mo + kWarps * GQA * D;                          // [warp][GQA] m, then l
  float* ml = mm + kWarps * GQA;
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
#pragma unroll
    for (int j = 0; j < C::CPL; ++j) mo[(warp * GQA + h) * D + lane * C::CPL + j] = o[h][j];
    if (lane == 0) { mm[warp * GQA + h] = m[h]; ml[warp * GQA + h] = l[h]; }
  }
  __syncthreads();
  float* dst = a.part + (int64_t)item * GQA * (2 + D);
  for (int i = threadIdx.x; i < GQA * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = NEG_INF;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w * GQA + h]);
    float acc = 0.f, L = 0.f;
    if (M != NEG_INF) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = mm[w * GQA + h];
        const float wt = mw == NEG_INF ? 0.f : exp2f(mw - M);
        acc = fmaf(wt, mo[(w * GQA + h) * D + d], acc);
        L = fmaf(wt, ml[w * GQA + h], L);
      }
    }
    dst[h * (2 + D) + 2 + d] = acc;
    if (d == 0) { dst[h * (2 + D)] = M; dst[h * (2 + D) + 1] = L; }
  }
}

// out[unit, h, d] = LSE merge of the unit's ns partials
template <int D, int GQA>
__global__ void merge_kernel(const __grid_constant__ Args a) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  const int unit = blockIdx.x;
  const int bh = unit % a.BH, layer = unit / a.BH;
  const int b = bh / a.HKV, kvh = bh % a.HKV;
  const float* src = a.part + (int64_t)unit * a.ns * GQA * (2 + D);
  for (int i = threadIdx.x; i < GQA * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = NEG_INF;
    for (int s = 0; s < a.ns; ++s) M = fmaxf(M, src[(s * GQA + h) * (2 + D)]);
    float acc = 0.f, L = 0.f;
    if (M != NEG_INF) {
      for (int s = 0; s < a.ns; ++s) {
        const float* ps = src + (s * GQA + h) * (2 + D);
        if (ps[0] == NEG_INF) continue;
        const float wt = exp2f(ps[0] - M);
        acc = fmaf(wt, ps[2 + d], acc);
        L = fmaf(wt, ps[1], L);
      }
    }
    const float r = L > 0.f ? acc / L : 0.f;
    const int64_t row = (int64_t)b * a.HQ + kvh * GQA + h;
    if (a.out_f32) static_cast<float*>(a.L[layer].out)[row * D + d] = r;
    else static_cast<uint16_t*>(a.L[layer].out)[row * D + d] = f32_to_bf16_bits(r);
  }
}

static int splits_for(const kvr_decode_args* a, int sms) {
  const int nch = (a->seq_len + kChunk - 1) / kChunk;
  if (a->split_tokens > 0) {
    const int cps = std::max(1, (a->split_tokens + kChunk - 1) / kChunk);
    return (nch + cps - 1) / cps;
  }
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  // about 4 resident CTAs per SM, and at least 8 chunks (2 per warp) per split
  const int64_t want = std::max<int64_t>(1, (4LL * sms + units - 1) / units);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, std::max(1, nch / 8)));
}

static size_t workspace_bytes(const kvr_decode_args* a, int ns) {
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  const int gqa = a->q_heads / a->kv_heads;
  return (size_t)units * ns * gqa * (2 + a->head_dim) * sizeof(float);
}

template <int D, int KB, int VB, int GQA>
static int run_t(const kvr_decode_args* a, int ns, cudaStream_t stream) {
  using C = SCfg<D, KB, VB, GQA>;
  static bool attr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KVR_ERR_CUDA;
  if (!attr[dev & 63]) {
    const cudaError_t e = cudaFuncSetAttribute(partial_kernel<D, KB, VB, GQA>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    attr[dev & 63] = true;
  }
  Args p;
  for (int l = 0; l < a->n_layers; ++l) {
    const kvr_layer_ptrs& L = a->layers[l];
    p.L[l] = Layer{L.key_payload, L.key_scale, L.key_offset, L.key_residual, L.value_payload,
                   L.value_scale, L.value_offset, L.query, L.out};
  }
  p.BH = a->batch * a->kv_heads;
  p.HKV = a->kv_heads;
  p.HQ = a->q_heads;
  p.S = a->seq_len;
  p.P = a->prefix_len;
  int lg = 0;
  while ((1 << lg) < a->group_size) ++lg;
  p.log2G = lg;
  p.ns = ns;
  const int nch = (a->seq_len + kChunk - 1) / kChunk;
  p.cps = (nch + ns - 1) / ns;
  p.out_f32 = a->out_dtype == 1;
  p.kp_bh = a->key_payload_bh_stride;
  p.km_bh = a->key_meta_bh_stride;
  p.kr_bh = a->key_residual_bh_stride;
  p.vp_bh = a->value_payload_bh_stride;
  p.vm_bh = a->value_meta_bh_stride;
  p.cs = (float)(1.4426950408889634 / std::sqrt((double)D));
  p.part = static_cast<float*>(a->workspace);
  const int64_t units = (int64_t)a->n_layers * p.BH;
  partial_kernel<D, KB, VB, GQA><<<(unsigned)(units * ns), kWarps * 32, C::SMEM, stream>>>(p);
  const int st = check_launch();
  if (st != KVR_OK) return st;
  merge_kernel<D, GQA><<<(unsigned)units, 128, 0, stream>>>(p);
  return check_launch();
}

static int validate(const kvr_decode_args* a) {
  if (!a || !a->layers || a->n_layers < 1 || a->n_layers > KVR_MAX_LAYERS || a->batch < 1 || a->kv_heads < 1 ||
      a->q_heads % a->kv_heads || a->seq_len < 1 || a->prefix_len < 0 || a->prefix_len > a->seq_len ||
      a->group_size < 32 || (a->group_size & (a->group_size - 1)) || a->prefix_len % a->group_size ||
      a->out_dtype < 0 || a->out_dtype > 1)
    return KVR_ERR_INVALID_ARGUMENT;
  for (int l = 0; l < a->n_layers; ++l) {
    const kvr_layer_ptrs& L = a->layers[l];
    if (!L.value_payload || !L.value_scale || !L.value_offset || !L.query || !L.out) return KVR_ERR_INVALID_ARGUMENT;
    if (a->prefix_len > 0 && (!L.key_payload || !L.key_scale || !L.key_offset)) return KVR_ERR_INVALID_ARGUMENT;
    if (a->prefix_len < a->seq_len && !L.key_residual) return KVR_ERR_INVALID_ARGUMENT;
    if ((L.key_payload && !aligned16(L.key_payload)) || (L.key_residual && !aligned16(L.key_residual)))
      return KVR_ERR_MISALIGNED;
  }
  return KVR_OK;
}

// (D, key bits, value bits, HQ/HKV) instantiated below
static bool supported(const kvr_decode_args* a) {
  const int g = a->q_heads / a->kv_heads;
  const int c[5][4] = {{128, 4, 4, 6}, {128, 2, 2, 6}, {128, 4, 4, 4}, {64, 8, 4, 4}, {64, 4, 8, 4}};
  for (const auto& x : c)
    if (a->head_dim == x[0] && a->key_bits == x[1] && a->value_bits == x[2] && g == x[3]) return true;
  return false;
}

static int device_sms(const kvr_decode_args* a) {
  if (a->num_sms > 0) return a->num_sms;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace simt
}  // namespace kvr

using namespace kvr;

extern "C" size_t kvr_decode_simt_workspace(const kvr_decode_args* a) {
  if (simt::validate(a) != KVR_OK || !simt::supported(a)) return 0;
  return simt::workspace_bytes(a, simt::splits_for(a, simt::device_sms(a)));
}

extern "C" int kvr_decode_attention_simt(const kvr_decode_args* a, kvr_stream_t stream) {
  const int st = simt::validate(a);
  if (st != KVR_OK) return st;
  if (!simt::supported(a)) return KVR_ERR_UNSUPPORTED;
  const int ns = simt::splits_for(a, simt::device_sms(a));
  if (!a->workspace || a->workspace_bytes < simt::workspace_bytes(a, ns)) return KVR_ERR_WORKSPACE;
  if (!aligned16(a->workspace)) return KVR_ERR_MISALIGNED;
  const int gqa = a->q_heads / a->kv_heads;
  cudaStream_t s = as_stream(stream);
#define KVR_SIMT_CASE(D_, KB_, VB_, G_)                                                              \
  if (a->head_dim == D_ && a->key_bits == KB_ && a->value_bits == VB_ && gqa == G_)                  \
    return simt::run_t<D_, KB_, VB_, G_>(a, ns, s);
  KVR_SIMT_CASE(128, 4, 4, 6) KVR_SIMT_CASE(128, 2, 2, 6) KVR_SIMT_CASE(128, 4, 4, 4)
  KVR_SIMT_CASE(64, 8, 4, 4) KVR_SIMT_CASE(64, 4, 8, 4)
#undef KVR_SIMT_CASE
  return KVR_ERR_UNSUPPORTED;
}
