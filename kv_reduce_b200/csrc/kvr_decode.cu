// Split-K decode attention over the bit-packed KIVI cache (sm_100a).
//
// Replaces the three Triton kernels of kv_reduce/triton_packed_kv_attention.py
// (:27-131 single pass, :134-248 split, :251-281 LSE reduce) with one launch:
//
//   grid  = layers x (batch*kv_heads) x splits, 4 warps per CTA
//   warp  = independent streamer of 32-token chunks through a private
//           3-stage cp.async ring in shared memory (16-byte copies, rows
//           XOR-swizzled so the tensor-core operand reads are conflict free)
//   QK^T  = mma.sync m16n8k16, M = 16 tokens, N = 8 query heads of the GQA
//           group (each packed byte is read once for all heads), K = head dim.
//           Key codes are turned into exact fp16 integers in registers with
//           the 0x6400 magic-exponent method (code | 0x6400 is 1024+code),
//           the per-channel key scale is folded into the fp16 query
//           (q~ = q * s_g * log2e/sqrt(D)), the zero point into a per-group
//           bias  q . z_g  computed in fp32.
//   softmax = fp32 online softmax in log2 units with warp-shuffle reductions.
//   P V    = mma.sync with M = head dim, N = heads, K = 16 tokens: P is moved
//           from accumulator to operand layout with movmatrix.trans, value
//           codes arrive token-paired through ldmatrix.trans, the per-token
//           value scale is folded into P (P~ = p * s_t) and the value zero
//           point is accumulated as sum(p * z_t) in fp32.
//   BF16 residual window = same pass, bf16 mma of raw keys against the raw
//           bf16 query (exact products).
//   epilogue = CTA merge of the 4 warps in shared memory, then the last CTA
//           of each (layer, b, kv head) merges the split partials (LSE merge)
//           and writes the output; its counter is reset for the next launch.
#include "kvr_common.cuh"

#include <algorithm>
#include <cmath>

namespace kvr {
namespace dec {

constexpr int kChunk = 32;    // tokens per pipeline stage
constexpr int kWarps = 4;     // warps per CTA
constexpr int kStages = 3;    // cp.async ring depth per warp
constexpr int kHeads = 8;     // N of the mma = padded GQA group
constexpr int kMaxSplits = 256;
constexpr uint32_t kMagic = 0x64006400u;  // fp16x2 {1024, 1024}

template <int D, int KB, int VB>
struct Cfg {
  static constexpr int RBK = D * KB / 8;  // key payload bytes per token
  static constexpr int RBV = D * VB / 8;  // value payload bytes per token
  static constexpr int CRK = RBK / 16;    // 16-byte pieces per key row
  static constexpr int CRV = RBV / 16;
  static constexpr int KS = D / 16;       // QK k-steps == PV m-tiles
  static constexpr int BT = RBK / 4;      // key bytes read per thread per row
  static constexpr int NWK = BT / 4;      // ... as 32-bit words
  static constexpr int RPWK = 2 * (8 / KB);  // fp16x2 registers per key word
  static constexpr int CPB_V = 16 / VB;   // value codes per b16 of an ldmatrix row
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = kChunk * RBK;
  static constexpr int M_OFF = V_OFF + kChunk * RBV;
  static constexpr int META = 4 * D;      // scale + offset bf16 for one group
  static constexpr int STAGE = M_OFF + 2 * META;   // two group slots
  static constexpr int RING = kStages * STAGE;
  static constexpr int MERGE = kWarps * kHeads * (D + 2) * 4;
  static constexpr int SMEM = (kWarps * RING > MERGE ? kWarps * RING : MERGE) + kMaxSplits * kHeads * 4;
  static_assert(CRK >= 1 && CRK <= 8 && (CRK & (CRK - 1)) == 0, "key row must be 16..128 bytes");
  static_assert(CRV >= 2 && CRV <= 8 && (CRV & (CRV - 1)) == 0, "value row must be 32..128 bytes");
  static_assert(D / 8 == (D / 4 * KB / 8 / 4) * RPWK, "key register count");
};

// XOR swizzle of the 16-byte piece index within a row: rows of CR pieces,
// 8/CR rows per 128 bytes, so eight consecutive rows at the same logical
// piece land in eight different bank quads.
template <int CR>
__device__ __forceinline__ int swz(int row) {
  if constexpr (CR == 1) return 0;
  else return (row / (8 / CR)) % CR;
}

struct LayerPtrs {
  const uint8_t* kp;
  const uint16_t* ks;
  const uint16_t* ko;
  const uint16_t* kr;
  const uint8_t* vp;
  const uint16_t* vs;
  const uint16_t* vo;
  const uint16_t* q;
  uint16_t* out;
};

template <int MAXL>
struct Params {
  LayerPtrs L[MAXL];
  int n_layers, BH, HQ, HKV, gqa;
  int S, P, G;
  int tok_begin, tok_end;        // token range processed (multiple of 32 begin)
  int num_splits, chunks_per_split;
  int64_t kp_bh, km_bh, kr_bh, vp_bh, vm_bh;
  float score_scale_log2;        // log2(e) / sqrt(D)
  float* part;                   // split partials (num_splits > 1)
  int* counters;                 // one per (layer, bh), zero on entry/exit
  float* out_ml;                 // partial mode: (m, l) per (layer, b, hq)
  float* out_o;                  // partial mode: unnormalised o
};

// Register-level conversions ------------------------------------------------
// Key register r of a thread: d_local = (r / RPW) * (32/KB) + r % RPW + e * (16/KB),
// scale factor 2^(KB * (j % (8/KB))), j = r % RPW.
template <int KB>
__device__ __forceinline__ constexpr int kb_rpw() { return 2 * (8 / KB); }
template <int KB>
__device__ __forceinline__ constexpr int key_dlocal(int r, int e) {
  return (r / kb_rpw<KB>()) * (32 / KB) + (r % kb_rpw<KB>()) + e * (16 / KB);
}
template <int B>
__device__ __forceinline__ constexpr float code_factor(int j) {
  return (float)(1u << (B * (j % (8 / B))));
}
template <int B>
__device__ __forceinline__ constexpr uint32_t code_mask(int j) {
  return ((((1u << B) - 1u) << (B * (j % (8 / B)))) * 0x00010001u);
}
// Exact fp16x2 {c_lo * f, c_hi * f} of code slot j of the two 16-bit halves.
template <int B>
__device__ __forceinline__ uint32_t codes_to_h2(uint32_t w, int j) {
  const uint32_t x = (j / (8 / B)) ? (w >> 8) : w;
  return hsub2_u32(lop_and_or(x, code_mask<B>(j), kMagic), kMagic);
}

template <int D, int KB, int VB, int MAXL>
__global__ void __launch_bounds__(kWarps * 32, 3) decode_kernel(const __grid_constant__ Params<MAXL> p) {
  using C = Cfg<D, KB, VB>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;

  const int NS = p.num_splits;
  const int sp = blockIdx.x % NS;
  const int rest = blockIdx.x / NS;
  const int bh = rest % p.BH;
  const int layer = rest / p.BH;
  const LayerPtrs& Lp = p.L[layer];
  const int b = bh / p.HKV, kvh = bh % p.HKV;
  const int S = p.S, P = p.P, G = p.G;
  const int t_end = p.tok_end;

  const uint8_t* kp = Lp.kp + (int64_t)bh * p.kp_bh;
  const uint16_t* ksc = Lp.ks + (int64_t)bh * p.km_bh;
  const uint16_t* kof = Lp.ko + (int64_t)bh * p.km_bh;
  const uint16_t* kres = Lp.kr + (int64_t)bh * p.kr_bh;
  const uint8_t* vp = Lp.vp + (int64_t)bh * p.vp_bh;
  const uint16_t* vsc = Lp.vs + (int64_t)bh * p.vm_bh;
  const uint16_t* vof = Lp.vo + (int64_t)bh * p.vm_bh;

  // ---------------------------------------------------------------- query
  // Thread (g, t4) owns head g of the group and head-dim slice
  // [t4*D/4, (t4+1)*D/4).  qcf = q * log2e/sqrt(D) / factor, per key register.
  const bool head_ok = g < p.gqa;
  const uint16_t* qrow = Lp.q + ((int64_t)b * p.HQ + kvh * p.gqa + (head_ok ? g : 0)) * D;
  const int dbase = t4 * (D / 4);
  float qcf[D / 8][2];
#pragma unroll
  for (int r = 0; r < D / 8; ++r)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float qv = head_ok ? bf16_bits_to_f32(qrow[dbase + key_dlocal<KB>(r, e)]) : 0.f;
      qcf[r][e] = qv * p.score_scale_log2 / code_factor<KB>(r % C::RPWK);
    }

  // ---------------------------------------------------------- chunk range
  const int c_first = p.tok_begin / kChunk;
  const int c_all = (t_end - p.tok_begin + kChunk - 1) / kChunk;
  const int c0 = c_first + sp * p.chunks_per_split;
  const int c1 = c_first + min(c_all, (sp + 1) * p.chunks_per_split);
  const int my_n = (c1 - c0 - warp + kWarps - 1) / kWarps > 0 ? (c1 - c0 - warp + kWarps - 1) / kWarps : 0;

  uint8_t* ring = smem + warp * C::RING;
  const uint32_t ring_s = smem_u32(ring);

  auto chunk_of = [&](int i) { return c0 + warp + i * kWarps; };

  auto issue = [&](int c, int stage) {
    const int tok0 = c * kChunk;
    const int n_valid = min(kChunk, t_end - tok0);
    const int n_pref = max(0, min(n_valid, P - tok0));
    const uint32_t st = ring_s + stage * C::STAGE;
    for (int pc = lane; pc < n_pref * C::CRK; pc += 32) {
      const int row = pc / C::CRK, c16 = pc % C::CRK;
      cp_async16(st + C::K_OFF + row * C::RBK + 16 * (c16 ^ swz<C::CRK>(row)),
                 kp + (int64_t)(tok0 + row) * C::RBK + 16 * c16);
    }
    for (int pc = lane; pc < n_valid * C::CRV; pc += 32) {
      const int row = pc / C::CRV, c16 = pc % C::CRV;
      cp_async16(st + C::V_OFF + row * C::RBV + 16 * (c16 ^ swz<C::CRV>(row)),
                 vp + (int64_t)(tok0 + row) * C::RBV + 16 * c16);
    }
    if (n_pref > 0) {
      const int g0 = tok0 / G;
      const int g1 = (n_pref > 16) ? (tok0 + 16) / G : g0;
      const int pieces = D / 8;   // 16-byte pieces of one D-long bf16 vector
      for (int pc = lane; pc < 4 * pieces; pc += 32) {
        const int slot = pc / (2 * pieces);
        const int which = (pc / pieces) & 1;   // 0 scale, 1 offset
        const int k16 = pc % pieces;
        if (slot == 1 && g1 == g0) continue;
        const int grp = slot ? g1 : g0;
        const uint16_t* src = (which ? kof : ksc) + (int64_t)grp * D + 8 * k16;
        cp_async16(st + C::M_OFF + slot * C::META + which * 2 * D + 16 * k16, src);
      }
    }
  };

  auto load_vmeta = [&](int c) -> uint32_t {
    const int t = c * kChunk + lane;
    if (t < t_end) return (uint32_t)__ldg(vsc + t) | ((uint32_t)__ldg(vof + t) << 16);
    return 0u;
  };

  // ------------------------------------------------------------ state
  float acc[C::KS][4];
#pragma unroll
  for (int i = 0; i < C::KS; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const float NEG_INF = -__int_as_float(0x7f800000);
  float m_run[2] = {NEG_INF, NEG_INF};
  float l_run[2] = {0.f, 0.f};
  float z_run[2] = {0.f, 0.f};
  uint32_t qt[D / 8];
  float bias[2] = {0.f, 0.f};
  int cur_grp = -1;

  // --------------------------------------------------------------- prologue
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (i < my_n) issue(chunk_of(i), i);
    cp_async_commit();
  }
  uint32_t vm_next = my_n > 0 ? load_vmeta(chunk_of(0)) : 0u;

  for (int i = 0; i < my_n; ++i) {
    {
      const int inext = i + kStages - 1;
      if (inext < my_n) issue(chunk_of(inext), inext % kStages);
      cp_async_commit();
    }
    const uint32_t vm_cur = vm_next;
    if (i + 1 < my_n) vm_next = load_vmeta(chunk_of(i + 1));
    cp_async_wait<kStages - 1>();
    __syncwarp();

    const int c = chunk_of(i);
    const int tok0 = c * kChunk;
    const int n_valid = min(kChunk, t_end - tok0);
    const uint8_t* st = ring + (i % kStages) * C::STAGE;
    const uint32_t st_s = ring_s + (i % kStages) * C::STAGE;

    // ------------------------------------------------------------- Q K^T
    float sc[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int mtok = tok0 + 16 * mt;
      sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
      if (16 * mt >= n_valid) {
        sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = NEG_INF;
        continue;
      }
      if (mtok < P) {
        const int grp = mtok / G;
        if (grp != cur_grp) {
          // q~ and bias for this key group (scale/offset from the stage).
          const int slot = (mt == 1 && grp != tok0 / G) ? 1 : 0;
          const uint16_t* sv = reinterpret_cast<const uint16_t*>(st + C::M_OFF + slot * C::META);
          const uint16_t* zv = sv + D;
          uint32_t sw[D / 8], zw[D / 8];
#pragma unroll
          for (int v = 0; v < D / 32; ++v) {
            const uint4 a = *reinterpret_cast<const uint4*>(sv + dbase + 8 * v);
            const uint4 z = *reinterpret_cast<const uint4*>(zv + dbase + 8 * v);
            sw[4 * v + 0] = a.x; sw[4 * v + 1] = a.y; sw[4 * v + 2] = a.z; sw[4 * v + 3] = a.w;
            zw[4 * v + 0] = z.x; zw[4 * v + 1] = z.y; zw[4 * v + 2] = z.z; zw[4 * v + 3] = z.w;
          }
          float bsum = 0.f;
#pragma unroll
          for (int r = 0; r < D / 8; ++r) {
            float qq[2];
            float part = 0.f;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int dl = key_dlocal<KB>(r, e);
              const float s = (dl & 1) ? bf16hi(sw[dl >> 1]) : bf16lo(sw[dl >> 1]);
              const float z = (dl & 1) ? bf16hi(zw[dl >> 1]) : bf16lo(zw[dl >> 1]);
              qq[e] = qcf[r][e] * s;
              part = fmaf(qcf[r][e], z, part);
            }
            qt[r] = pack_half2(qq[0], qq[1]);
            bsum = fmaf(part, code_factor<KB>(r % C::RPWK), bsum);
          }
          bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
          bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
          bias[0] = __shfl_sync(0xffffffffu, bsum, 4 * (2 * t4));
          bias[1] = __shfl_sync(0xffffffffu, bsum, 4 * (2 * t4 + 1));
          cur_grp = grp;
        }
        // key words of rows 16mt+g and 16mt+g+8, thread slice [t4*BT, +BT)
        uint32_t kw[2][C::NWK];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = 16 * mt + g + 8 * h;
          const uint8_t* rowp = st + C::K_OFF + row * C::RBK;
          if constexpr (C::BT >= 16) {
#pragma unroll
            for (int v = 0; v < C::BT / 16; ++v) {
              const int c16 = (t4 * C::BT) / 16 + v;
              const uint4 x = *reinterpret_cast<const uint4*>(rowp + 16 * (c16 ^ swz<C::CRK>(row)));
              kw[h][4 * v + 0] = x.x; kw[h][4 * v + 1] = x.y; kw[h][4 * v + 2] = x.z; kw[h][4 * v + 3] = x.w;
            }
          } else if constexpr (C::BT == 8) {
            const int lb = t4 * 8;
            const uint2 x = *reinterpret_cast<const uint2*>(rowp + 16 * ((lb >> 4) ^ swz<C::CRK>(row)) + (lb & 15));
            kw[h][0] = x.x; kw[h][1] = x.y;
          } else {
            const int lb = t4 * 4;
            kw[h][0] = *reinterpret_cast<const uint32_t*>(rowp + 16 * ((lb >> 4) ^ swz<C::CRK>(row)) + (lb & 15));
          }
        }
        float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int js = 0; js < C::KS; ++js) {
          const int r0 = 2 * js, r1 = 2 * js + 1;
          const uint32_t a0 = codes_to_h2<KB>(kw[0][r0 / C::RPWK], r0 % C::RPWK);
          const uint32_t a1 = codes_to_h2<KB>(kw[1][r0 / C::RPWK], r0 % C::RPWK);
          const uint32_t a2 = codes_to_h2<KB>(kw[0][r1 / C::RPWK], r1 % C::RPWK);
          const uint32_t a3 = codes_to_h2<KB>(kw[1][r1 / C::RPWK], r1 % C::RPWK);
          mma_f16(a4, a0, a1, a2, a3, qt[r0], qt[r1]);
        }
        sc[mt][0] = a4[0] + bias[0];
        sc[mt][1] = a4[1] + bias[1];
        sc[mt][2] = a4[2] + bias[0];
        sc[mt][3] = a4[3] + bias[1];
      } else {
        // BF16 residual window: raw keys x raw query, bf16 mma.
        uint32_t kr[2][D / 8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = mtok + g + 8 * h;
          if (tok < t_end) {
            const uint4* src = reinterpret_cast<const uint4*>(kres + (int64_t)(tok - P) * D + dbase);
#pragma unroll
            for (int v = 0; v < D / 32; ++v) {
              const uint4 x = __ldg(src + v);
              kr[h][4 * v + 0] = x.x; kr[h][4 * v + 1] = x.y; kr[h][4 * v + 2] = x.z; kr[h][4 * v + 3] = x.w;
            }
          } else {
#pragma unroll
            for (int v = 0; v < D / 8; ++v) kr[h][v] = 0u;
          }
        }
        uint32_t qb[D / 8];
        {
          const uint4* src = reinterpret_cast<const uint4*>(qrow + dbase);
#pragma unroll
          for (int v = 0; v < D / 32; ++v) {
            uint4 x = __ldg(src + v);
            if (!head_ok) x = make_uint4(0u, 0u, 0u, 0u);
            qb[4 * v + 0] = x.x; qb[4 * v + 1] = x.y; qb[4 * v + 2] = x.z; qb[4 * v + 3] = x.w;
          }
        }
        float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int js = 0; js < C::KS; ++js)
          mma_bf16(a4, kr[0][2 * js], kr[1][2 * js], kr[0][2 * js + 1], kr[1][2 * js + 1], qb[2 * js], qb[2 * js + 1]);
#pragma unroll
        for (int k = 0; k < 4; ++k) sc[mt][k] = a4[k] * p.score_scale_log2;
      }
      // mask tokens past the end
      if (mtok + g >= t_end) { sc[mt][0] = NEG_INF; sc[mt][1] = NEG_INF; }
      if (mtok + g + 8 >= t_end) { sc[mt][2] = NEG_INF; sc[mt][3] = NEG_INF; }
    }

    // ---------------------------------------------------------- softmax
    float cmax[2];
    cmax[0] = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
    cmax[1] = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      cmax[0] = fmaxf(cmax[0], __shfl_xor_sync(0xffffffffu, cmax[0], o));
      cmax[1] = fmaxf(cmax[1], __shfl_xor_sync(0xffffffffu, cmax[1], o));
    }
    const bool grow = (cmax[0] > m_run[0]) || (cmax[1] > m_run[1]);
    if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float mn = fmaxf(m_run[e], cmax[e]);
        const float alpha = (mn == NEG_INF) ? 1.f : fast_exp2(m_run[e] - mn);
        m_run[e] = mn;
        l_run[e] *= alpha;
        z_run[e] *= alpha;
#pragma unroll
        for (int mi = 0; mi < C::KS; ++mi) {
          acc[mi][e] *= alpha;
          acc[mi][2 + e] *= alpha;
        }
      }
    }
    uint32_t pb[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t vm_lo = __shfl_sync(0xffffffffu, vm_cur, 16 * mt + g);
      const uint32_t vm_hi = __shfl_sync(0xffffffffu, vm_cur, 16 * mt + g + 8);
      const float s_lo = bf16lo(vm_lo), z_lo = bf16hi(vm_lo);
      const float s_hi = bf16lo(vm_hi), z_hi = bf16hi(vm_hi);
      float pr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float mref = m_run[k & 1];
        pr[k] = (sc[mt][k] == NEG_INF) ? 0.f : fast_exp2(sc[mt][k] - mref);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l_run[e] += pr[e] + pr[2 + e];
        z_run[e] = fmaf(pr[e], z_lo, fmaf(pr[2 + e], z_hi, z_run[e]));
      }
      pb[mt][0] = movmatrix_trans(pack_half2(pr[0] * s_lo, pr[1] * s_lo));
      pb[mt][1] = movmatrix_trans(pack_half2(pr[2] * s_hi, pr[3] * s_hi));
    }

    // ---------------------------------------------------------------- P V
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      if (16 * ks >= n_valid) break;
      uint32_t vx[2][C::CRV];
#pragma unroll
      for (int q4 = 0; q4 < C::CRV / 2; ++q4) {
        const int m = 4 * q4 + (lane >> 3);
        const int blk = m / C::CRV, c16 = m % C::CRV;
        const int row = 16 * ks + 8 * blk + (lane & 7);
        const uint32_t addr = st_s + C::V_OFF + row * C::RBV + 16 * (c16 ^ swz<C::CRV>(row));
        uint32_t r0, r1, r2, r3;
        ldsm_x4_trans(addr, r0, r1, r2, r3);
        const int mb = 4 * q4;
        vx[(mb + 0) / C::CRV][(mb + 0) % C::CRV] = r0;
        vx[(mb + 1) / C::CRV][(mb + 1) % C::CRV] = r1;
        vx[(mb + 2) / C::CRV][(mb + 2) % C::CRV] = r2;
        vx[(mb + 3) / C::CRV][(mb + 3) % C::CRV] = r3;
      }
#pragma unroll
      for (int mi = 0; mi < C::KS; ++mi) {
        const int ra = 2 * mi, rb = 2 * mi + 1;
        const uint32_t a0 = codes_to_h2<VB>(vx[0][ra / C::CPB_V], ra % C::CPB_V);
        const uint32_t a1 = codes_to_h2<VB>(vx[0][rb / C::CPB_V], rb % C::CPB_V);
        const uint32_t a2 = codes_to_h2<VB>(vx[1][ra / C::CPB_V], ra % C::CPB_V);
        const uint32_t a3 = codes_to_h2<VB>(vx[1][rb / C::CPB_V], rb % C::CPB_V);
        mma_f16(acc[mi], a0, a1, a2, a3, pb[ks][0], pb[ks][1]);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  // ------------------------------------------------------ warp finalisation
#pragma unroll
  for (int e = 0; e < 2; ++e) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], o);
      z_run[e] += __shfl_xor_sync(0xffffffffu, z_run[e], o);
    }
  }
  __syncthreads();   // ring no longer needed: reuse as merge area
  float* mO = reinterpret_cast<float*>(smem);                 // [W][8][D]
  float* mM = mO + kWarps * kHeads * D;                      // [W][8]
  float* mL = mM + kWarps * kHeads;                           // [W][8]
#pragma unroll
  for (int mi = 0; mi < C::KS; ++mi) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 2 * mi + hh;
      const int cch = r / C::CPB_V, j = r % C::CPB_V;
      const int d = cch * (128 / VB) + g * C::CPB_V + j;
      const float inv = 1.f / code_factor<VB>(j);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int h = 2 * t4 + e;
        mO[(warp * kHeads + h) * D + d] = fmaf(acc[mi][2 * hh + e], inv, z_run[e]);
      }
    }
  }
  if (g == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mM[warp * kHeads + 2 * t4 + e] = m_run[e];
      mL[warp * kHeads + 2 * t4 + e] = l_run[e];
    }
  }
  __syncthreads();

  // ------------------------------------------------------- CTA merge (warps)
  const int gqa = p.gqa;
  const bool partial_mode = p.out_ml != nullptr;
  const int64_t unit = (int64_t)layer * p.BH + bh;
  float* part = NS > 1 ? p.part + (unit * NS + sp) * (int64_t)(kHeads * (D + 2)) : nullptr;
  for (int idx = threadIdx.x; idx < gqa * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    float M = NEG_INF;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mM[w * kHeads + h]);
    float o = 0.f, l = 0.f;
    if (M != NEG_INF) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = mM[w * kHeads + h];
        if (mw == NEG_INF) continue;
        const float wt = fast_exp2(mw - M);
        o = fmaf(wt, mO[(w * kHeads + h) * D + d], o);
        l = fmaf(wt, mL[w * kHeads + h], l);
      }
    }
    if (NS == 1) {
      const int64_t row = (int64_t)b * p.HQ + kvh * gqa + h;
      if (partial_mode) {
        const int64_t prow = (int64_t)layer * (p.BH / p.HKV) * p.HQ + row;
        p.out_o[prow * D + d] = o;
        if (d == 0) { p.out_ml[2 * prow] = M; p.out_ml[2 * prow + 1] = l; }
      } else {
        Lp.out[row * D + d] = f32_to_bf16_bits(l > 0.f ? o / l : 0.f);
      }
    } else {
      part[2 * kHeads + h * D + d] = o;
      if (d == 0) { part[h] = M; part[kHeads + h] = l; }
    }
  }
  if (NS == 1) return;

  // -------------------------------------------- split merge by the last CTA
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.counters + unit, 1) == NS - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* wts = reinterpret_cast<float*>(smem + C::SMEM - kMaxSplits * kHeads * 4);  // [NS][8]
  __shared__ float s_M[kHeads], s_L[kHeads];
  const float* base = p.part + unit * NS * (int64_t)(kHeads * (D + 2));
  const int64_t pstride = kHeads * (D + 2);
  for (int h = warp; h < gqa; h += kWarps) {
    float M = NEG_INF;
    for (int s = lane; s < NS; s += 32) M = fmaxf(M, __ldcg(base + s * pstride + h));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int s = lane; s < NS; s += 32) {
      const float ms = __ldcg(base + s * pstride + h);
      const float wt = (ms == NEG_INF || M == NEG_INF) ? 0.f : fast_exp2(ms - M);
      wts[s * kHeads + h] = wt;
      L = fmaf(wt, __ldcg(base + s * pstride + kHeads + h), L);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) { s_M[h] = M; s_L[h] = L; }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < gqa * (D / 4); idx += blockDim.x) {
    const int h = idx / (D / 4), d = 4 * (idx % (D / 4));
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = base + 2 * kHeads + h * D + d;
#pragma unroll 4
    for (int s = 0; s < NS; ++s) {
      const float wt = wts[s * kHeads + h];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + s * pstride));
      o.x = fmaf(wt, v.x, o.x); o.y = fmaf(wt, v.y, o.y);
      o.z = fmaf(wt, v.z, o.z); o.w = fmaf(wt, v.w, o.w);
    }
    const float M = s_M[h], L = s_L[h];
    const int64_t row = (int64_t)b * p.HQ + kvh * gqa + h;
    if (partial_mode) {
      const int64_t prow = (int64_t)layer * (p.BH / p.HKV) * p.HQ + row;
      *reinterpret_cast<float4*>(p.out_o + prow * D + d) = o;
      if (d == 0) { p.out_ml[2 * prow] = M; p.out_ml[2 * prow + 1] = L; }
    } else {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      uint2 w;
      w.x = (uint32_t)f32_to_bf16_bits(o.x * inv) | ((uint32_t)f32_to_bf16_bits(o.y * inv) << 16);
      w.y = (uint32_t)f32_to_bf16_bits(o.z * inv) | ((uint32_t)f32_to_bf16_bits(o.w * inv) << 16);
      *reinterpret_cast<uint2*>(Lp.out + row * D + d) = w;
    }
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;
}

// LSE merge of externally produced partials (cross-GPU token split).
__global__ void lse_merge_kernel(const float* __restrict__ ml, const float* __restrict__ o, int n_parts,
                                 int rows, int D, uint16_t* __restrict__ out) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)rows * D;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / D;
    float M = NEG_INF;
    for (int pp = 0; pp < n_parts; ++pp) M = fmaxf(M, ml[2 * ((int64_t)pp * rows + row)]);
    float acc = 0.f, L = 0.f;
    if (M != NEG_INF) {
      for (int pp = 0; pp < n_parts; ++pp) {
        const float mp = ml[2 * ((int64_t)pp * rows + row)];
        if (mp == NEG_INF) continue;
        const float wt = exp2f(mp - M);
        acc = fmaf(wt, o[((int64_t)pp * rows) * D + i], acc);
        L = fmaf(wt, ml[2 * ((int64_t)pp * rows + row) + 1], L);
      }
    }
    out[i] = f32_to_bf16_bits(L > 0.f ? acc / L : 0.f);
  }
}

// ------------------------------------------------------------------ host
struct Plan {
  int num_splits = 1, chunks_per_split = 1;
  size_t counters = 0, part_bytes = 0;
};

static int device_sms(int hint) {
  if (hint > 0) return hint;
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  }
  return n;
}

static Plan make_plan(const kvr_decode_args* a, int tok_begin, int tok_end) {
  Plan pl;
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  const int nchunks = std::max(1, (tok_end - tok_begin + kChunk - 1) / kChunk);
  int cps;
  if (a->split_tokens > 0) {
    cps = (a->split_tokens + kChunk - 1) / kChunk;
  } else {
    const int sms = device_sms(a->num_sms);
    const int64_t target = (int64_t)sms * 3;   // ~one wave at 3 CTAs per SM
    int ns = (int)std::max<int64_t>(1, (target + units - 1) / units);
    cps = (nchunks + ns - 1) / ns;
    cps = std::max(cps, 2 * kWarps);            // at least two chunks per warp
  }
  cps = std::max(cps, 1);
  int ns = (nchunks + cps - 1) / cps;
  if (ns > kMaxSplits) {
    cps = (nchunks + kMaxSplits - 1) / kMaxSplits;
    ns = (nchunks + cps - 1) / cps;
  }
  pl.num_splits = ns;
  pl.chunks_per_split = cps;
  pl.counters = (size_t)units;
  pl.part_bytes = ns > 1 ? (size_t)units * ns * kHeads * (a->head_dim + 2) * 4 : 0;
  return pl;
}

static int validate(const kvr_decode_args* a) {
  if (!a || !a->layers || a->n_layers < 1 || a->n_layers > KVR_MAX_LAYERS) return KVR_ERR_INVALID_ARGUMENT;
  if (a->batch < 1 || a->kv_heads < 1 || a->q_heads < 1 || a->q_heads % a->kv_heads) return KVR_ERR_INVALID_ARGUMENT;
  if (a->q_heads / a->kv_heads > kHeads) return KVR_ERR_UNSUPPORTED;
  if (a->head_dim != 64 && a->head_dim != 128) return KVR_ERR_UNSUPPORTED;
  auto bits_ok = [](int b) { return b == 2 || b == 4 || b == 8; };
  if (!bits_ok(a->key_bits) || !bits_ok(a->value_bits)) return KVR_ERR_UNSUPPORTED;
  if (a->head_dim == 64 && a->value_bits == 2) return KVR_ERR_UNSUPPORTED;
  if (a->seq_len < 1 || a->prefix_len < 0 || a->prefix_len > a->seq_len) return KVR_ERR_INVALID_ARGUMENT;
  if (a->group_size <= 0 || a->group_size % 16) return KVR_ERR_UNSUPPORTED;
  if (a->prefix_len % a->group_size) return KVR_ERR_INVALID_ARGUMENT;
  if (a->key_payload_bh_stride % 16 || a->value_payload_bh_stride % 16 || a->key_meta_bh_stride % 8 ||
      a->key_residual_bh_stride % 8)
    return KVR_ERR_MISALIGNED;
  for (int l = 0; l < a->n_layers; ++l) {
    const kvr_layer_ptrs& L = a->layers[l];
    if (!L.value_payload || !L.value_scale || !L.value_offset || !L.query || !L.out) return KVR_ERR_INVALID_ARGUMENT;
    if (a->prefix_len > 0 && (!L.key_payload || !L.key_scale || !L.key_offset)) return KVR_ERR_INVALID_ARGUMENT;
    if (a->prefix_len < a->seq_len && !L.key_residual) return KVR_ERR_INVALID_ARGUMENT;
    if ((L.key_payload && !aligned16(L.key_payload)) || !aligned16(L.value_payload) ||
        (L.key_scale && !aligned16(L.key_scale)) || (L.key_offset && !aligned16(L.key_offset)) ||
        (L.key_residual && !aligned16(L.key_residual)) || !aligned16(L.query))
      return KVR_ERR_MISALIGNED;
  }
  return KVR_OK;
}

template <int MAXL>
static void fill_params(Params<MAXL>& p, const kvr_decode_args* a, const Plan& pl, int tb, int te) {
  for (int l = 0; l < a->n_layers; ++l) {
    const kvr_layer_ptrs& L = a->layers[l];
    p.L[l] = LayerPtrs{L.key_payload, L.key_scale, L.key_offset, L.key_residual, L.value_payload,
                       L.value_scale, L.value_offset, L.query, L.out};
  }
  p.n_layers = a->n_layers;
  p.BH = a->batch * a->kv_heads;
  p.HQ = a->q_heads;
  p.HKV = a->kv_heads;
  p.gqa = a->q_heads / a->kv_heads;
  p.S = a->seq_len;
  p.P = a->prefix_len;
  p.G = a->group_size;
  p.tok_begin = tb;
  p.tok_end = te;
  p.num_splits = pl.num_splits;
  p.chunks_per_split = pl.chunks_per_split;
  p.kp_bh = a->key_payload_bh_stride;
  p.km_bh = a->key_meta_bh_stride;
  p.kr_bh = a->key_residual_bh_stride;
  p.vp_bh = a->value_payload_bh_stride;
  p.vm_bh = a->value_meta_bh_stride;
  p.score_scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)a->head_dim));
  p.counters = a->counters;
  p.part = pl.num_splits > 1 ? static_cast<float*>(a->workspace) : nullptr;
  p.out_ml = nullptr;
  p.out_o = nullptr;
}

template <int D, int KB, int VB, int MAXL>
static int launch_t(const Params<MAXL>& p, int grid, cudaStream_t s) {
  using C = Cfg<D, KB, VB>;
  auto kern = decode_kernel<D, KB, VB, MAXL>;
  static bool attr_done = false;   // per instantiation; benign race sets the same value
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    attr_done = true;
  }
  kern<<<grid, kWarps * 32, C::SMEM, s>>>(p);
  return check_launch();
}

template <int MAXL>
static int dispatch(const Params<MAXL>& p, const kvr_decode_args* a, int grid, cudaStream_t s) {
#define KVR_CASE(D_, KB_, VB_)                                                              \
  if (a->head_dim == D_ && a->key_bits == KB_ && a->value_bits == VB_)                      \
    return launch_t<D_, KB_, VB_, MAXL>(p, grid, s);
  KVR_CASE(128, 4, 4) KVR_CASE(128, 8, 4) KVR_CASE(128, 4, 8) KVR_CASE(128, 8, 8)
  KVR_CASE(128, 2, 2) KVR_CASE(128, 2, 4) KVR_CASE(128, 4, 2) KVR_CASE(128, 8, 2) KVR_CASE(128, 2, 8)
  KVR_CASE(64, 4, 4) KVR_CASE(64, 8, 4) KVR_CASE(64, 4, 8) KVR_CASE(64, 8, 8) KVR_CASE(64, 2, 4)
  KVR_CASE(64, 2, 8)
#undef KVR_CASE
  return KVR_ERR_UNSUPPORTED;
}

static int run(const kvr_decode_args* a, int tb, int te, float* out_ml, float* out_o, cudaStream_t s) {
  int st = validate(a);
  if (st != KVR_OK) return st;
  if (tb < 0 || te > a->seq_len || tb >= te || tb % kChunk) return KVR_ERR_INVALID_ARGUMENT;
  Plan pl = make_plan(a, tb, te);
  if (pl.num_splits > 1) {
    if (!a->workspace || a->workspace_bytes < pl.part_bytes || !a->counters) return KVR_ERR_WORKSPACE;
    if (!aligned16(a->workspace)) return KVR_ERR_MISALIGNED;
  }
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  const int64_t grid = units * pl.num_splits;
  if (grid > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  if (a->n_layers == 1) {
    Params<1> p;
    fill_params(p, a, pl, tb, te);
    p.out_ml = out_ml; p.out_o = out_o;
    return dispatch(p, a, (int)grid, s);
  }
  Params<KVR_MAX_LAYERS> p;
  fill_params(p, a, pl, tb, te);
  p.out_ml = out_ml; p.out_o = out_o;
  return dispatch(p, a, (int)grid, s);
}

}  // namespace dec
}  // namespace kvr

using namespace kvr;

extern "C" int kvr_decode_plan(const kvr_decode_args* a, int* num_splits, size_t* workspace_bytes,
                               size_t* counter_count) {
  int st = dec::validate(a);
  if (st != KVR_OK) return st;
  dec::Plan pl = dec::make_plan(a, 0, a->seq_len);
  if (num_splits) *num_splits = pl.num_splits;
  if (workspace_bytes) *workspace_bytes = pl.part_bytes;
  if (counter_count) *counter_count = pl.counters;
  return KVR_OK;
}

extern "C" int kvr_decode_attention(const kvr_decode_args* a, kvr_stream_t stream) {
  if (!a) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, 0, a->seq_len, nullptr, nullptr, as_stream(stream));
}

extern "C" int kvr_decode_partial(const kvr_decode_args* a, int token_begin, int token_end, float* part_ml,
                                  float* part_o, kvr_stream_t stream) {
  if (!a || !part_ml || !part_o) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, token_begin, token_end, part_ml, part_o, as_stream(stream));
}

extern "C" int kvr_lse_merge(const float* part_ml, const float* part_o, int n_parts, int rows, int head_dim,
                             uint16_t* out, kvr_stream_t stream) {
  if (!part_ml || !part_o || !out || n_parts < 1 || rows < 0 || head_dim < 1) return KVR_ERR_INVALID_ARGUMENT;
  if (rows == 0) return KVR_OK;
  const int64_t total = (int64_t)rows * head_dim;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  dec::lse_merge_kernel<<<grid, 256, 0, as_stream(stream)>>>(part_ml, part_o, n_parts, rows, head_dim, out);
  return check_launch();
}
