// Split-K decode attention over the bit-packed KIVI cache (sm_100a).
//
// Replaces the three Triton kernels of kv_reduce/triton_packed_kv_attention.py
// (:27-131 single pass, :134-248 split, :251-281 LSE reduce) with one launch:
//
//   work  = (layer, batch*kv_head, split) items; a persistent grid of
//           resident CTAs strides over them, the split count chosen by a
//           cost model so the last wave is full (kvr_decode_plan)
//   warp  = independent streamer of 32-token chunks through a private
//           2-stage cp.async ring in shared memory (16-byte copies, rows
//           XOR-swizzled so the tensor-core operand reads are conflict free)
//   QK^T  = mma.sync m16n8k16, M = 16 tokens, N = 8 query heads of the GQA
//           group (each packed byte is read once for all heads), K = head dim.
//           Key codes become exact fp16 subnormals in registers with one AND
//           (code bits in the mantissa of a zero exponent: c * f * 2^-24);
//           the per-channel key scale is folded into the query,
//           q~ = (q / f) * s_g (f = the code's bit-position factor), carried
//           as an exact fp16 hi + lo pair (TwoProduct); s_g comes as fp16
//           pairs in register order from a table written when the group was
//           packed (kvr_key_scale_pairs), or is converted from the bf16
//           scales per chunk when a cache has no table; the zero point
//           enters as a per-group bias q . z_g from a bf16 mma; scores are
//           scaled by 2^24 * log2e / sqrt(D) after the mma.
//   softmax = fp32 online softmax in log2 units with warp-shuffle reductions.
//   P V    = mma.sync with M = head dim, N = heads, K = 16 tokens: P moves
//           from accumulator to operand layout with movmatrix.trans, value
//           codes arrive token-paired through ldmatrix.trans and become
//           exact fp16 subnormals with one AND, as the keys do
//           (c * f * 2^-24, undone in the epilogue), the per-token value
//           scale is folded into P (P~ = p * s_t) and the zero point is
//           accumulated as sum p * z_t in fp32.
//   BF16 residual window = same pass, bf16 mma of raw keys against the raw
//           bf16 query (exact products).
//   epilogue = CTA merge of the 4 warps in shared memory, then a two-level
//           last-arriver LSE merge of the split partials (groups of 16), the
//           counters reset by the merging CTA for the next launch.
#include "kvr_common.cuh"

#include <type_traits>

#include <algorithm>
#include <atomic>
#include <cmath>

namespace kvr {
namespace dec {

constexpr int kChunk = 32;    // tokens per pipeline stage
constexpr int kWarps = 4;     // warps per CTA
constexpr int kStages = 2;    // cp.async ring depth per warp (one chunk ahead hides HBM latency)
constexpr int kHeads = 8;     // N of the mma = padded GQA group
constexpr int kMaxSplits = 256;
constexpr int kFan = 16;      // partials merged per merge step
static_assert(kFan <= 16, "a cluster of kFan CTAs must be launchable");
constexpr uint32_t kMagic = 0x64006400u;  // fp16x2 {1024, 1024}

template <int D, int KB, int VB>
struct Cfg {
  static constexpr int RBK = D * KB / 8;  // key payload bytes per token
  static constexpr int RBV = D * VB / 8;  // value payload bytes per token
  static constexpr int CRK = RBK / 16;    // 16-byte pieces per key row
  static constexpr int CRV = RBV / 16;
  static constexpr int KS = D / 16;       // QK k-steps == PV m-tiles
  static constexpr int BT = RBK / 4;      // key bytes read per thread per row
  static constexpr int NWK = BT >= 4 ? BT / 4 : 1;   // ... as 32-bit words
  static constexpr int RPWK = 2 * (8 / KB);   // fp16x2 registers per key word
  static constexpr int CPB_V = 16 / VB;   // value codes per b16 of an ldmatrix row
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = kChunk * RBK;
  static constexpr int M_OFF = V_OFF + kChunk * RBV;
  static constexpr int META = 4 * D;      // scale + offset bf16 for one group
  static constexpr int VM_OFF = M_OFF + 2 * META;  // value scale[32] then offset[32], bf16
  static constexpr int STAGE = VM_OFF + 2 * kChunk * 2;
  static constexpr int RING = kStages * STAGE;
  // staged query per lane: D/8 fp16x2 words in key-register order (q / f)
  // then the D/8 raw bf16x2 words of its head-dim slice, as uint4 [D/16][32]
  static constexpr int QS_OFF = kWarps * RING;
  static constexpr int QS_BYTES = (D / 16) * 32 * 16;
  static constexpr int MERGE = kWarps * kHeads * (D + 2) * 4;
  // cluster merge: this CTA's partial (M[8], L[8], o[8][D]) after the warp merge area
  static constexpr int CPART_OFF = (MERGE + 15) / 16 * 16;
  static constexpr int CPART_END = CPART_OFF + kHeads * (D + 2) * 4;
  static constexpr int BODY = QS_OFF + QS_BYTES;
  static constexpr int SMEM = BODY > CPART_END ? BODY : CPART_END;
  // resident CTAs per SM the register budget is sized for: 4 (16 warps) unless
  // 8-bit keys at D=128 need the registers of a 3-CTA budget
  static constexpr int MIN_CTAS = (KB == 8 && D == 128) ? 3 : 4;
  static_assert(CRK >= 1 && CRK <= 8 && (CRK & (CRK - 1)) == 0, "key row must be 16..128 bytes");
  static_assert(CRV >= 2 && CRV <= 8 && (CRV & (CRV - 1)) == 0, "value row must be 32..128 bytes");
  static_assert(D / 8 == NWK * RPWK, "key register count");
};

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
  void* out;
  const uint16_t* ksp;   // key scales as fp16 pairs in register order, or null
};

template <int MAXL>
struct Params {
  LayerPtrs L[MAXL];
  int n_layers, BH, HQ, HKV, gqa, batch;
  int S, P, G, log2G;
  int tok_begin, tok_end;        // token range processed (begin multiple of 32)
  int num_splits, chunks_per_split, items, groups1;
  int64_t kp_bh, km_bh, kr_bh, vp_bh, vm_bh;
  int vm_staged;                 // value scale/offset rows 16-byte aligned: copy them with the chunk
  float score_scale_log2;        // log2(e) / sqrt(D)
  int out_f32;                   // 1: fp32 output, 0: bf16
  float* part1;                  // [units][NS][pstride]
  float* part2;                  // [units][groups1][pstride]
  int* cnt1;                     // [units][groups1]
  int* cnt2;                     // [units]
  float* out_ml;                 // partial mode: (m, l) per (layer, b, hq)
  float* out_o;                  // partial mode: unnormalised o
  int* dev_len;                  // non-null: sequence / prefix length read here at run time
  int res_cap;                   // residual rows the key residual buffer holds
  int cluster;                   // > 1: launched in clusters of NS CTAs, one per unit
  int q_shared;                  // queries in host-mapped memory: in a cluster, rank 0 alone reads them
  // fused append of one new token per (b, kv head) before the decode
  // (device-side lengths only): its key row goes to the BF16 residual, its
  // value row is quantized per token, and the sequence length advances
  const uint16_t* app_k;         // [B, HKV, 1, D] bf16, or null
  const uint16_t* app_v;
  // fused sequence-split exchange (partial mode, kvr_decode_partial_exchange):
  // the partials of this launch go, as (value, epoch) words, to half
  // (epoch % 2), source slot x_rank, of every rank's receive area
  int* const* x_signal;          // device array [x_world]: signal areas (receive areas at +kLLWords), or null
  const int* x_epoch;            // exchanges completed on this rank; this step is *x_epoch + 1
  int x_world, x_rank;
  int x_owner;                   // 1: each row goes to its owner rank (row % x_world) only
};
constexpr int kLLWords = 64;     // 32-bit words of a signal area before its receive area

// Append one token of unit bh (one warp; lane = D/32 channels): the key row
// into the BF16 residual at res_row, the value row quantized per token into
// row s of the value payload and metadata -- the arithmetic of the append
// kernel (exact min/max, IEEE scale, affine_code_rcp), so the bytes match it.
template <int D, int VB, typename P>
__device__ __forceinline__ void append_token(const P& p, const LayerPtrs& Lp, int bh, int s, int res_row, int lane) {
  constexpr int K = D / 32;
  constexpr int LB = K * VB / 8;
  constexpr int levels = (1 << VB) - 1;
  const int64_t src = (int64_t)bh * D + lane * K;
  uint16_t* kr = const_cast<uint16_t*>(Lp.kr) + (int64_t)bh * p.kr_bh + (int64_t)res_row * D + lane * K;
  if constexpr (K == 2) *reinterpret_cast<uint32_t*>(kr) = *reinterpret_cast<const uint32_t*>(p.app_k + src);
  else *reinterpret_cast<uint2*>(kr) = *reinterpret_cast<const uint2*>(p.app_k + src);
  float xv[K];
  load_bf16x<K>(p.app_v + src, xv);
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
  const float scale = affine_scale(mn, mx, VB);
  const float inv = __frcp_rn(scale);
  uint64_t w = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) w |= (uint64_t)affine_code_rcp(xv[k], mn, scale, inv, levels) << (k * VB);
  store_bytes<LB>(const_cast<uint8_t*>(Lp.vp) + (int64_t)bh * p.vp_bh + (int64_t)s * (32 * LB) + lane * LB, w);
  if (lane == 0) {
    const int64_t m = (int64_t)bh * p.vm_bh + s;
    const_cast<uint16_t*>(Lp.vs)[m] = f32_to_bf16_bits(scale);
    const_cast<uint16_t*>(Lp.vo)[m] = f32_to_bf16_bits(mn);
  }
}

// ------------------------------------------------------- thread-block clusters
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t dsmem_map(uint32_t smem_addr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 dsmem_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}

// one 16-byte store of two (value, tag) words; volatile, so it is issued
// as written and each 8-byte half lands whole
__device__ __forceinline__ void st_volatile_v4(uint32_t* ptr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"l"(ptr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// ----------------------------------------------------------- register maps
// Key register r of a thread (head-dim slice [t4*D/4, +D/4)):
//   d_local(r, e) = (r / RPW) * (32/KB) + r % RPW + e * (16/KB),
//   scale factor 2^(KB * (j % (8/KB))) with j = r % RPW.
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
// fp16x2 {1024 + c*f} for the subtraction that leaves (code - c) * f.
template <int B>
__device__ __forceinline__ constexpr uint32_t sub_const(int j, bool centred) {
  // fp16 of 1024 + k with integer 0 <= k < 1024 is 0x6400 + k
  const uint32_t k = centred ? (1u << (B - 1)) * (1u << (B * (j % (8 / B)))) : 0u;
  return (0x6400u + k) * 0x00010001u;
}
// Exact fp16x2 {(c_lo - off) * f, (c_hi - off) * f} of code slot j of both halves.
template <int B, bool CENTRED>
__device__ __forceinline__ uint32_t codes_to_h2(uint32_t w, int j) {
  const uint32_t x = (j / (8 / B)) ? (w >> 8) : w;
  return hsub2_u32(lop_and_or(x, code_mask<B>(j), kMagic), sub_const<B>(j, CENTRED));
}

// Key code slot j of both halves as exact fp16x2 subnormals
// {c_lo * f * 2^-24, c_hi * f * 2^-24}: the masked code bits sit in the
// mantissa of a zero exponent field (f = 2^(B * (j % (8/B))) <= 64, so the
// value stays below 2^-14).  The tensor cores take fp16 subnormal operands
// exactly; the 2^-24 is folded into the score scale, so no subtraction of a
// magic-number bias is needed.
template <int B>
__device__ __forceinline__ uint32_t key_codes_h2(uint32_t w, int j) {
  const uint32_t x = (j / (8 / B)) ? (w >> 8) : w;
  return x & code_mask<B>(j);
}
// Sticky per-device flag: set when a decode emits a non-finite output
// (an fp16 tensor-core operand out of range: a key scale or q~ = q s / f
// at or above 65504 after the query scaling below, a value scale at or
// above 65504), read and cleared by kvr_decode_nonfinite.
__device__ unsigned int g_decode_nonfinite;
// Queries with |q| >= 2^kQueryExp are scaled by an exact power of two so
// |q| < 2^kQueryExp: q / f and q~ = q s / f then stay in fp16 range for key
// scales below 2^(15 - kQueryExp).  Scores are scaled back in fp32.
constexpr int kQueryExp = 6;
constexpr float kKeyUnscale = 16777216.f;          // 2^24
constexpr float kKeyScale = 1.f / 16777216.f;      // 2^-24

// Per-chunk state of one warp's query transform for a key group.
template <int D>
struct GroupQ {
  uint32_t hi[D / 8];
  uint32_t lo[D / 8];
  float bias[2];
};

// Per key group: q~ = (q / f) * s as an exact fp16 hi + lo pair (TwoProduct),
// and the zero-point bias  q . z  for heads 2*t4, 2*t4+1 from one bf16 mma
// per k-step whose A rows all hold z (exact bf16 products, fp32 sums), so the
// bias lands in the accumulator layout of the QK^T tiles.
template <int D, int KB>
__device__ __forceinline__ void group_query(GroupQ<D>& gq, const uint4* qs, const uint16_t* meta, int lane,
                                            int dbase, bool pairs) {
  uint32_t sw[D / 8];
#pragma unroll
  for (int v = 0; v < D / 32; ++v) {
    const uint4 a = *reinterpret_cast<const uint4*>(meta + dbase + 8 * v);
    sw[4 * v + 0] = a.x; sw[4 * v + 1] = a.y; sw[4 * v + 2] = a.z; sw[4 * v + 3] = a.w;
  }
#pragma unroll
  for (int v = 0; v < D / 32; ++v) {
    const uint4 qh = qs[v * 32 + lane];
    const uint32_t qw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = 4 * v + k;
      const int d0 = key_dlocal<KB>(r, 0), d1 = key_dlocal<KB>(r, 1);
      const float s0 = (d0 & 1) ? bf16hi(sw[d0 >> 1]) : bf16lo(sw[d0 >> 1]);
      const float s1 = (d1 & 1) ? bf16hi(sw[d1 >> 1]) : bf16lo(sw[d1 >> 1]);
      two_prod_h2(qw[k], pairs ? sw[r] : pack_half2(s0, s1), gq.hi[r], gq.lo[r]);
    }
  }
  float bf[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int v = 0; v < D / 32; ++v) {
    const uint4 z = *reinterpret_cast<const uint4*>(meta + D + dbase + 8 * v);
    const uint4 qb = qs[(D / 32 + v) * 32 + lane];
    mma_bf16(bf, z.x, z.x, z.y, z.y, qb.x, qb.y);
    mma_bf16(bf, z.z, z.z, z.w, z.w, qb.z, qb.w);
  }
  gq.bias[0] = bf[0];
  gq.bias[1] = bf[1];
}

// Key words of chunk row `row` for this thread's byte slice [t4*BT, +BT).
template <int D, int KB>
__device__ __forceinline__ void load_key_row(uint32_t (&kw)[Cfg<D, KB, 4>::NWK], const uint8_t* kbase, int row,
                                             int t4) {
  using C = Cfg<D, KB, 4>;
  const uint8_t* rowp = kbase + row * C::RBK;
  if constexpr (C::BT >= 16) {
#pragma unroll
    for (int v = 0; v < C::BT / 16; ++v) {
      const int c16 = (t4 * C::BT) / 16 + v;
      const uint4 x = *reinterpret_cast<const uint4*>(rowp + 16 * (c16 ^ swz<C::CRK>(row)));
      kw[4 * v + 0] = x.x; kw[4 * v + 1] = x.y; kw[4 * v + 2] = x.z; kw[4 * v + 3] = x.w;
    }
  } else if constexpr (C::BT == 8) {
    const int lb = t4 * 8;
    const uint2 x = *reinterpret_cast<const uint2*>(rowp + 16 * ((lb >> 4) ^ swz<C::CRK>(row)) + (lb & 15));
    kw[0] = x.x; kw[1] = x.y;
  } else {
    const int lb = t4 * 4;
    kw[0] = *reinterpret_cast<const uint32_t*>(rowp + 16 * ((lb >> 4) ^ swz<C::CRK>(row)) + (lb & 15));
  }
}

// Zero-point bias of a key group, q . z for heads 2*t4, 2*t4+1, from one bf16
// mma per k-step whose A rows all hold z; returned in accumulator layout.
template <int D>
__device__ __forceinline__ void group_bias(float (&bf)[4], const uint4* qs, const uint16_t* meta, int lane,
                                           int dbase) {
  bf[0] = bf[1] = bf[2] = bf[3] = 0.f;
#pragma unroll
  for (int v = 0; v < D / 32; ++v) {
    const uint4 z = *reinterpret_cast<const uint4*>(meta + D + dbase + 8 * v);
    const uint4 qb = qs[(D / 32 + v) * 32 + lane];
    mma_bf16(bf, z.x, z.x, z.y, z.y, qb.x, qb.y);
    mma_bf16(bf, z.z, z.z, z.w, z.w, qb.z, qb.w);
  }
}

// QK^T of a whole 32-token chunk inside one key group: rows g, g+8, g+16,
// g+24 in kw[0..3]; the hi/lo query for each k-step is formed on the fly
// from shared memory (s words and q/f words in windows), keeping the live
// register set small.  h0/h1 arrive holding the bias.
template <int D, int KB, bool PAIRS>
__device__ __forceinline__ void qk_chunk(float (&h0)[4], float (&l0)[4], float (&h1)[4], float (&l1)[4],
                                         const uint32_t (&kw)[4][D / 8 / (2 * (8 / KB))], const uint4* qs,
                                         const uint16_t* meta, int lane, int dbase) {
  constexpr int RPW = kb_rpw<KB>();
  constexpr int JPW = (KB == 2) ? 4 : 2;   // k-steps per window
  constexpr int WIN = 2 * JPW;             // s words per window (and q words)
  uint32_t sw[WIN], qw[WIN];
#pragma unroll
  for (int js = 0; js < D / 16; ++js) {
    if (js % JPW == 0) {
      const int m = js / JPW;
#pragma unroll
      for (int v = 0; v < WIN / 4; ++v) {
        const uint4 a = *reinterpret_cast<const uint4*>(meta + dbase + 2 * (WIN * m + 4 * v));
        sw[4 * v + 0] = a.x; sw[4 * v + 1] = a.y; sw[4 * v + 2] = a.z; sw[4 * v + 3] = a.w;
        const uint4 q = qs[(WIN * m / 4 + v) * 32 + lane];
        qw[4 * v + 0] = q.x; qw[4 * v + 1] = q.y; qw[4 * v + 2] = q.z; qw[4 * v + 3] = q.w;
      }
    }
    const int base = WIN * (js / JPW);   // first register / word of the window
    uint32_t bh[2], bl[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = 2 * js + k;
      uint32_t sp;
      if constexpr (PAIRS) {
        sp = sw[r - base];   // the pair of register r, converted when the group was packed
      } else {
        const int d0 = key_dlocal<KB>(r, 0), d1 = key_dlocal<KB>(r, 1);
        const int w0 = (d0 >> 1) - base, w1 = (d1 >> 1) - base;
        const float s0 = (d0 & 1) ? bf16hi(sw[w0]) : bf16lo(sw[w0]);
        const float s1 = (d1 & 1) ? bf16hi(sw[w1]) : bf16lo(sw[w1]);
        sp = pack_half2(s0, s1);
      }
      two_prod_h2(qw[r - base], sp, bh[k], bl[k]);
    }
    const int r0 = 2 * js, r1 = 2 * js + 1;
    const uint32_t a0 = key_codes_h2<KB>(kw[0][r0 / RPW], r0 % RPW);
    const uint32_t a1 = key_codes_h2<KB>(kw[1][r0 / RPW], r0 % RPW);
    const uint32_t a2 = key_codes_h2<KB>(kw[0][r1 / RPW], r1 % RPW);
    const uint32_t a3 = key_codes_h2<KB>(kw[1][r1 / RPW], r1 % RPW);
    const uint32_t b0 = key_codes_h2<KB>(kw[2][r0 / RPW], r0 % RPW);
    const uint32_t b1 = key_codes_h2<KB>(kw[3][r0 / RPW], r0 % RPW);
    const uint32_t b2 = key_codes_h2<KB>(kw[2][r1 / RPW], r1 % RPW);
    const uint32_t b3 = key_codes_h2<KB>(kw[3][r1 / RPW], r1 % RPW);
    mma_f16(h0, a0, a1, a2, a3, bh[0], bh[1]);
    mma_f16(h1, b0, b1, b2, b3, bh[0], bh[1]);
    mma_f16(l0, a0, a1, a2, a3, bl[0], bl[1]);
    mma_f16(l1, b0, b1, b2, b3, bl[0], bl[1]);
  }
}

// QK^T of one prefix m-tile: rows (tokens) g and g+8 from kw0 / kw1.
template <int D, int KB>
__device__ __forceinline__ void qk_prefix(float (&hi)[4], float (&lo)[4], const uint32_t* kw0, const uint32_t* kw1,
                                          const GroupQ<D>& gq) {
  constexpr int RPW = kb_rpw<KB>();
#pragma unroll
  for (int js = 0; js < D / 16; ++js) {
    const int r0 = 2 * js, r1 = 2 * js + 1;
    const uint32_t a0 = key_codes_h2<KB>(kw0[r0 / RPW], r0 % RPW);
    const uint32_t a1 = key_codes_h2<KB>(kw1[r0 / RPW], r0 % RPW);
    const uint32_t a2 = key_codes_h2<KB>(kw0[r1 / RPW], r1 % RPW);
    const uint32_t a3 = key_codes_h2<KB>(kw1[r1 / RPW], r1 % RPW);
    mma_f16(hi, a0, a1, a2, a3, gq.hi[r0], gq.hi[r1]);
    mma_f16(lo, a0, a1, a2, a3, gq.lo[r0], gq.lo[r1]);
  }
}

// XCHG: the fused-exchange instantiation (kvr_decode_partial_exchange); the
// others compile its stores and flag releases out
template <int D, int KB, int VB, int MAXL, bool XCHG = false>
__global__ void __launch_bounds__(kWarps * 32, Cfg<D, KB, VB>::MIN_CTAS) decode_kernel(const __grid_constant__ Params<MAXL> p) {
  using C = Cfg<D, KB, VB>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_flag;
  __shared__ int s_xe;   // fused exchange: this step's epoch
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int dbase = t4 * (D / 4);
  const float NEG_INF = -__int_as_float(0x7f800000);
  const int NS = p.num_splits;
  const int log2G = p.log2G;
  pdl_wait();   // nothing above touches global memory
  // the exchange of the previous step completed before pdl_wait returned,
  // so its epoch update is visible; read once, used after the CTA barriers
  if (XCHG && threadIdx.x == 0) s_xe = p.x_signal ? *reinterpret_cast<const volatile int*>(p.x_epoch) + 1 : 0;
  // Lengths: from the launch, or (graph-replayable loops) from device memory,
  // clamped to the capacities the host validated: sequence <= tok_end,
  // prefix <= P in whole groups, residual rows <= res_cap.
  int P = p.P, t_end = p.tok_end;
  int s_new = -1, res_new = 0;   // fused append: the new token's row and residual row
  if (p.dev_len) {
    const int dl_s = *reinterpret_cast<const volatile int*>(p.dev_len);
    const int dl_p = *reinterpret_cast<const volatile int*>(p.dev_len + 1);
    int S = dl_s;
    if (p.app_k) {
      // room for the token, as the append kernel checks it; a step past a
      // capacity sets the error flag and decodes without appending
      const bool ok = dl_p >= 0 && dl_p <= dl_s && dl_s + 1 <= p.tok_end && dl_s - dl_p + 1 <= p.res_cap;
      if (ok) {
        s_new = dl_s;
        res_new = dl_s - dl_p;
        S = dl_s + 1;
      }
      if (threadIdx.x == 0) {
        if (!ok && blockIdx.x == 0) atomicOr(p.dev_len + 2, 1);
        // every CTA has read the lengths before the last one advances them
        __threadfence();
        if (atomicAdd(p.dev_len + 3, 1) == (int)gridDim.x - 1) {
          p.dev_len[3] = 0;
          if (ok) p.dev_len[0] = S;
        }
      }
    }
    P = min(max(dl_p, 0), p.P) >> log2G << log2G;
    t_end = min(min(max(S, P), p.tok_end), P + p.res_cap);
  }
  uint8_t* ring = smem + warp * C::RING;
  const uint32_t ring_s = smem_u32(ring);
  uint4* qs = reinterpret_cast<uint4*>(smem + C::QS_OFF);
  __shared__ int s_qexp;                 // this item's query exponent shift

  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int sp = item % NS;
    const int unit = item / NS;
    const int bh = unit % p.BH;
    const int layer = unit / p.BH;
    const LayerPtrs& Lp = p.L[layer];
    const int b = bh / p.HKV, kvh = bh % p.HKV;
    const uint8_t* kp = Lp.kp + (int64_t)bh * p.kp_bh;
    // key scales: the fp16 pair table when the cache has one (same layout
    // and bytes as the bf16 scales), else the bf16 scales, converted per chunk
    const bool pairs = Lp.ksp != nullptr;
    const uint16_t* ksc = (pairs ? Lp.ksp : Lp.ks) + (int64_t)bh * p.km_bh;
    const uint16_t* kof = Lp.ko + (int64_t)bh * p.km_bh;
    const uint16_t* kres = Lp.kr + (int64_t)bh * p.kr_bh;
    const uint8_t* vp = Lp.vp + (int64_t)bh * p.vp_bh;
    const uint16_t* vsc = Lp.vs + (int64_t)bh * p.vm_bh;
    const uint16_t* vof = Lp.vo + (int64_t)bh * p.vm_bh;
    const bool head_ok = g < p.gqa;
    const uint16_t* qrow = Lp.q + ((int64_t)b * p.HQ + kvh * p.gqa + (head_ok ? g : 0)) * D;

    __syncthreads();   // previous item's merge area (aliases the rings) is dead
    if (s_new >= 0 && sp == (s_new / kChunk - p.tok_begin / kChunk) / p.chunks_per_split) {
      // this split holds the new token: store it before any chunk is read
      if (warp == 0) append_token<D, VB>(p, Lp, bh, s_new, res_new, lane);
      __threadfence();
      __syncthreads();
    }

    // ---------------------------------------------------------- chunk range
    const int c_first = p.tok_begin / kChunk;
    const int c_all = (t_end - p.tok_begin + kChunk - 1) / kChunk;
    const int c0 = c_first + sp * p.chunks_per_split;
    const int c1 = c_first + min(c_all, (sp + 1) * p.chunks_per_split);
    const int my_n = c1 - c0 > warp ? (c1 - c0 - warp + kWarps - 1) / kWarps : 0;

    auto issue = [&](int c, int stage) {
      const int tok0 = c * kChunk;
      const int n_valid = min(kChunk, t_end - tok0);
      const int n_pref = max(0, min(n_valid, P - tok0));
      const uint32_t st = ring_s + stage * C::STAGE;
      if (n_pref == kChunk && log2G >= 5) {
        // Full prefix chunk in one key group (the common case).  Piece k of
        // this lane sits at row lane/CR + k*32/CR, byte (lane%CR)*16, and its
        // swizzle term ((row / (8/CR)) % CR) reduces to (lane/8 + 4k) % CR, so
        // every copy is a per-lane base plus a compile-time offset.
        const uint8_t* ks = kp + (int64_t)tok0 * C::RBK + 16 * lane;
        const uint8_t* vs = vp + (int64_t)tok0 * C::RBV + 16 * lane;
        const uint32_t kd = st + C::K_OFF + (lane / C::CRK) * C::RBK +
                            16 * ((lane % C::CRK) ^ ((lane >> 3) & (C::CRK - 1)));
        const uint32_t vd = st + C::V_OFF + (lane / C::CRV) * C::RBV +
                            16 * ((lane % C::CRV) ^ ((lane >> 3) & (C::CRV - 1)));
#pragma unroll
        for (int k = 0; k < C::CRK; ++k)
          cp_async16(((C::CRK == 8 && (k & 1)) ? (kd ^ 64u) : kd) + 512 * k, ks + 512 * k);
#pragma unroll
        for (int k = 0; k < C::CRV; ++k)
          cp_async16(((C::CRV == 8 && (k & 1)) ? (vd ^ 64u) : vd) + 512 * k, vs + 512 * k);
        if (lane < D / 4) {   // key scale (lanes < D/8) and offset of the group, slot 0
          const int which = lane / (D / 8), k16 = lane % (D / 8);
          cp_async16(st + C::M_OFF + which * 2 * D + 16 * k16,
                     (which ? kof : ksc) + (int64_t)(tok0 >> log2G) * D + 8 * k16);
        }
        if (p.vm_staged && lane < 8)
          cp_async16(st + C::VM_OFF + (lane >> 2) * 2 * kChunk + 16 * (lane & 3),
                     ((lane >> 2) ? vof : vsc) + tok0 + 8 * (lane & 3));
        return;
      }
      const uint8_t* ksrc = kp + (int64_t)tok0 * C::RBK;
      const uint8_t* vsrc = vp + (int64_t)tok0 * C::RBV;
#pragma unroll
      for (int k = 0; k < C::CRK; ++k) {
        const int pc = lane + 32 * k;
        const int row = pc / C::CRK, c16 = pc % C::CRK;
        if (row < n_pref)
          cp_async16(st + C::K_OFF + row * C::RBK + 16 * (c16 ^ swz<C::CRK>(row)), ksrc + 16 * pc);
      }
#pragma unroll
      for (int k = 0; k < C::CRV; ++k) {
        const int pc = lane + 32 * k;
        const int row = pc / C::CRV, c16 = pc % C::CRV;
        if (row < n_valid)
          cp_async16(st + C::V_OFF + row * C::RBV + 16 * (c16 ^ swz<C::CRV>(row)), vsrc + 16 * pc);
      }
      if (p.vm_staged && lane < 8) {
        // 8 pieces: value scale then value offset, 8 tokens each; only whole
        // pieces inside the chunk (a ragged tail is read directly when used)
        const int k16 = lane & 3;
        if (8 * k16 + 8 <= n_valid)
          cp_async16(st + C::VM_OFF + (lane >> 2) * 2 * kChunk + 16 * k16, ((lane >> 2) ? vof : vsc) + tok0 + 8 * k16);
      }
      if (n_pref > 0) {
        // group slots: 0 <- group of rows 0..15, 1 <- group of rows 16..31 if different
        const int g0 = tok0 >> log2G;
        const int g1 = (n_pref > 16) ? ((tok0 + 16) >> log2G) : g0;
        constexpr int PIECES = D / 8;   // 16-byte pieces of a D-long bf16 vector
#pragma unroll
        for (int k = 0; k < (4 * PIECES + 31) / 32; ++k) {
          const int pc = lane + 32 * k;
          if (pc < 4 * PIECES) {
            const int slot = pc / (2 * PIECES);
            const int which = (pc / PIECES) & 1;
            const int k16 = pc % PIECES;
            if (slot == 0 || g1 != g0) {
              const int grp = slot ? g1 : g0;
              const uint16_t* src = (which ? kof : ksc) + (int64_t)grp * D + 8 * k16;
              cp_async16(st + C::M_OFF + slot * C::META + which * 2 * D + 16 * k16, src);
            }
          }
        }
      }
    };

    // value scale and offset of the lane's token, raw bf16 (scale | offset << 16).
    // Issued one chunk ahead and only converted when used, so the global
    // load latency hides behind a whole chunk of work.
    auto load_vmeta = [&](int c) -> uint32_t {
      const int t = c * kChunk + lane;
      uint32_t s = 0u, z = 0u;
      if (!p.vm_staged && t < t_end) {
        s = __ldg(vsc + t);
        z = __ldg(vof + t);
      }
      return s | (z << 16);
    };

    // -------------------------------------------------------------- state
    float acc[C::KS][4];
#pragma unroll
    for (int i = 0; i < C::KS; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m_run[2] = {NEG_INF, NEG_INF};
    float l_run[2] = {0.f, 0.f};
    float z_run[2] = {0.f, 0.f};

#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) {
      if (i < my_n) issue(c0 + warp + i * kWarps, i);
      cp_async_commit();
    }
    uint32_t vm_next = my_n > 0 ? load_vmeta(c0 + warp) : 0u;
    int stage = 0;

    // ------------------------------------- query -> shared memory (warp 0)
    // while the first chunks are in flight.  Lane (g, t4): words [0, D/8)
    // are fp16x2 (q[d(r,0)], q[d(r,1)]) / f_r in key-register order, words
    // [D/8, D/4) the raw bf16 pairs of q[dbase .. dbase + D/4).
    // Queries in host-mapped memory, clustered plan (one item per CTA, the
    // cluster = the unit's splits): rank 0 alone reads them across PCIe and
    // stages them; the other CTAs copy its staged words over distributed
    // shared memory, so each query crosses PCIe once, not once per split.
    const bool q_from_rank0 = p.q_shared && NS > 1 && p.cluster > 1;
    if (warp == 0 && !(q_from_rank0 && cluster_rank() != 0)) {
      uint32_t raw[D / 8];
      float amax = 0.f;
#pragma unroll
      for (int v = 0; v < D / 32; ++v) {
        uint4 x = head_ok ? __ldg(reinterpret_cast<const uint4*>(qrow + dbase) + v) : make_uint4(0u, 0u, 0u, 0u);
        raw[4 * v + 0] = x.x; raw[4 * v + 1] = x.y; raw[4 * v + 2] = x.z; raw[4 * v + 3] = x.w;
      }
#pragma unroll
      for (int w = 0; w < D / 8; ++w) amax = fmaxf(amax, fmaxf(fabsf(bf16lo(raw[w])), fabsf(bf16hi(raw[w]))));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      // |q| >= 2^kQueryExp: scale the query by 2^-qe (exact) so |q| < 2^kQueryExp
      const int qe = amax >= (float)(1 << kQueryExp) ? min(ilogbf(amax) - kQueryExp + 1, 120) : 0;
      const float qscale = __int_as_float((127 - qe) << 23);   // 2^-qe, exact
      if (lane == 0) s_qexp = qe;
#pragma unroll
      for (int v = 0; v < D / 32; ++v) {
        uint32_t wb[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t x = raw[4 * v + k];
          wb[k] = qe ? ((uint32_t)f32_to_bf16_bits(bf16lo(x) * qscale) |
                        ((uint32_t)f32_to_bf16_bits(bf16hi(x) * qscale) << 16))
                     : x;
        }
        qs[(D / 32 + v) * 32 + lane] = make_uint4(wb[0], wb[1], wb[2], wb[3]);
      }
#pragma unroll
      for (int v = 0; v < D / 32; ++v) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int r = 4 * v + k;
          const int d0 = key_dlocal<KB>(r, 0), d1 = key_dlocal<KB>(r, 1);
          const float inv = qscale / code_factor<KB>(r % C::RPWK);
          const float q0 = ((d0 & 1) ? bf16hi(raw[d0 >> 1]) : bf16lo(raw[d0 >> 1])) * inv;
          const float q1 = ((d1 & 1) ? bf16hi(raw[d1 >> 1]) : bf16lo(raw[d1 >> 1])) * inv;
          w[k] = pack_half2(q0, q1);
        }
        qs[v * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (q_from_rank0) {
      cluster_sync_all();   // rank 0's staged query and exponent are written and visible
      if (cluster_rank() != 0) {
        // rank 0 keeps them unchanged to the end of its item, and cannot end
        // it before this CTA reaches the cluster merge's barrier
        const uint32_t src = dsmem_map(smem_u32(qs), 0);
        for (int i = threadIdx.x; i < C::QS_BYTES / 16; i += blockDim.x) {
          const float4 v = dsmem_f32x4(src + 16 * i);
          qs[i] = make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
        }
        if (threadIdx.x == 0) s_qexp = __float_as_int(dsmem_f32(dsmem_map(smem_u32(&s_qexp), 0)));
      }
    }
    __syncthreads();
    // score scales of this item: log2(e)/sqrt(D), times the query's 2^qe;
    // quantized-key scores also carry the codes' 2^-24
    const float cs = p.score_scale_log2 * __int_as_float((127 + s_qexp) << 23);
    const float cs_k = cs * kKeyUnscale;

    for (int i = 0; i < my_n; ++i) {
      {
        const int inext = i + kStages - 1;
        int snext = stage + kStages - 1;
        if (snext >= kStages) snext -= kStages;
        if (inext < my_n) issue(c0 + warp + inext * kWarps, snext);
        cp_async_commit();
      }
      const uint32_t vm_cur = vm_next;
      if (i + 1 < my_n) vm_next = load_vmeta(c0 + warp + (i + 1) * kWarps);
      cp_async_wait<kStages - 1>();
      __syncwarp();

      const int c = c0 + warp + i * kWarps;
      const int tok0 = c * kChunk;
      const int n_valid = min(kChunk, t_end - tok0);
      const uint8_t* st = ring + stage * C::STAGE;
      const uint32_t st_s = ring_s + stage * C::STAGE;
      const uint16_t* meta0 = reinterpret_cast<const uint16_t*>(st + C::M_OFF);

      // A full prefix chunk inside one key group (the common case) runs a
      // body free of row bounds logic; other chunks take the general body.
      auto chunk_body = [&](auto full_c, auto pairs_c) {
        constexpr bool FULL = decltype(full_c)::value;
        constexpr bool PAIRS = decltype(pairs_c)::value;   // FULL body only
        // ------------------------------------------------------------ Q K^T
        float sc[2][4];
        if constexpr (FULL) {
          // whole chunk in one key group: both m-tiles, four independent mma chains
          // the hi chains start from the zero-point bias
          float bf[4];
          group_bias<D>(bf, qs, meta0, lane, dbase);
          uint32_t kw[4][C::NWK];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) load_key_row<D, KB>(kw[rr], st + C::K_OFF, g + 8 * rr, t4);
#pragma unroll
          for (int k = 0; k < 4; ++k) bf[k] *= kKeyScale;
          float h0[4] = {bf[0], bf[1], bf[2], bf[3]}, l0[4] = {0.f, 0.f, 0.f, 0.f};
          float h1[4] = {bf[0], bf[1], bf[2], bf[3]}, l1[4] = {0.f, 0.f, 0.f, 0.f};
          qk_chunk<D, KB, PAIRS>(h0, l0, h1, l1, kw, qs, meta0, lane, dbase);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            sc[0][k] = (h0[k] + l0[k]) * cs_k;
            sc[1][k] = (h1[k] + l1[k]) * cs_k;
          }
        } else {
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int mtok = tok0 + 16 * mt;
            sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = NEG_INF;
            if (16 * mt >= n_valid) continue;
            if (mtok < P) {
              const int grp = mtok >> log2G;
              const int slot = (mt == 1 && grp != (tok0 >> log2G)) ? 1 : 0;
              GroupQ<D> gq;
              group_query<D, KB>(gq, qs, meta0 + slot * (C::META / 2), lane, dbase, pairs);
              uint32_t kw0[C::NWK], kw1[C::NWK];
              load_key_row<D, KB>(kw0, st + C::K_OFF, 16 * mt + g, t4);
              load_key_row<D, KB>(kw1, st + C::K_OFF, 16 * mt + g + 8, t4);
              const float b0 = gq.bias[0] * kKeyScale, b1 = gq.bias[1] * kKeyScale;
              float hi[4] = {b0, b1, b0, b1}, lo[4] = {0.f, 0.f, 0.f, 0.f};
              qk_prefix<D, KB>(hi, lo, kw0, kw1, gq);
#pragma unroll
              for (int k = 0; k < 4; ++k) sc[mt][k] = (hi[k] + lo[k]) * cs_k;
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
#pragma unroll
              for (int v = 0; v < D / 32; ++v) {
                const uint4 x = qs[(D / 32 + v) * 32 + lane];
                qb[4 * v + 0] = x.x; qb[4 * v + 1] = x.y; qb[4 * v + 2] = x.z; qb[4 * v + 3] = x.w;
              }
              float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int js = 0; js < C::KS; ++js)
                mma_bf16(a4, kr[0][2 * js], kr[1][2 * js], kr[0][2 * js + 1], kr[1][2 * js + 1], qb[2 * js],
                         qb[2 * js + 1]);
#pragma unroll
              for (int k = 0; k < 4; ++k) sc[mt][k] = a4[k] * cs;
            }
            if (mtok + g >= t_end) { sc[mt][0] = NEG_INF; sc[mt][1] = NEG_INF; }
            if (mtok + g + 8 >= t_end) { sc[mt][2] = NEG_INF; sc[mt][3] = NEG_INF; }
          }
        }

        // ------------------------------------------------------------ softmax
        float cmax[2];
        cmax[0] = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
        cmax[1] = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
        // The running maxima can only move if some lane's own rows exceed
        // them; otherwise the reduced maxima would not either, so the
        // reduction and the rescale are skipped (bit-identical either way).
        const bool grow = (cmax[0] > m_run[0]) || (cmax[1] > m_run[1]);
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            cmax[0] = fmaxf(cmax[0], __shfl_xor_sync(0xffffffffu, cmax[0], o));
            cmax[1] = fmaxf(cmax[1], __shfl_xor_sync(0xffffffffu, cmax[1], o));
          }
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
          // token scale s and offset z of rows g, g+8
          uint32_t w_lo, w_hi;
          if (p.vm_staged) {
            const uint16_t* vm = reinterpret_cast<const uint16_t*>(st + C::VM_OFF);
            const int r = 16 * mt + g;
            if constexpr (FULL) {
              w_lo = (uint32_t)vm[r] | ((uint32_t)vm[kChunk + r] << 16);
              w_hi = (uint32_t)vm[r + 8] | ((uint32_t)vm[kChunk + r + 8] << 16);
            } else {
              // rows [0, n_vm) were copied; the ragged tail [n_vm, n_valid) is
              // read from global memory; rows past the end contribute zero
              const int n_vm = n_valid & ~7;
              auto vmeta = [&](int rr) -> uint32_t {
                if (rr < n_vm) return (uint32_t)vm[rr] | ((uint32_t)vm[kChunk + rr] << 16);
                if (rr < n_valid) return (uint32_t)__ldg(vsc + tok0 + rr) | ((uint32_t)__ldg(vof + tok0 + rr) << 16);
                return 0u;
              };
              w_lo = vmeta(r);
              w_hi = vmeta(r + 8);
            }
          } else {
            w_lo = __shfl_sync(0xffffffffu, vm_cur, 16 * mt + g);
            w_hi = __shfl_sync(0xffffffffu, vm_cur, 16 * mt + g + 8);
          }
          const float s_lo = bf16lo(w_lo), s_hi = bf16lo(w_hi);
          const float z_lo = bf16hi(w_lo), z_hi = bf16hi(w_hi);
          float pr[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) pr[k] = fast_exp2(sc[mt][k] - m_run[k & 1]);   // -inf -> 0
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
          if constexpr (!FULL) {
            if (16 * ks >= n_valid) break;
          }
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
            const uint32_t a0 = key_codes_h2<VB>(vx[0][ra / C::CPB_V], ra % C::CPB_V);
            const uint32_t a1 = key_codes_h2<VB>(vx[0][rb / C::CPB_V], rb % C::CPB_V);
            const uint32_t a2 = key_codes_h2<VB>(vx[1][ra / C::CPB_V], ra % C::CPB_V);
            const uint32_t a3 = key_codes_h2<VB>(vx[1][rb / C::CPB_V], rb % C::CPB_V);
            mma_f16(acc[mi], a0, a1, a2, a3, pb[ks][0], pb[ks][1]);
          }
        }
      };
      if ((n_valid == kChunk) && (tok0 + kChunk <= P) && (log2G >= 5)) {
        if (pairs) chunk_body(std::true_type{}, std::true_type{});
        else chunk_body(std::true_type{}, std::false_type{});
      } else {
        chunk_body(std::false_type{}, std::false_type{});
      }
      __syncwarp();
      stage = stage + 1 == kStages ? 0 : stage + 1;
    }
    cp_async_wait<0>();
    // the next kernel may be scheduled while the splits merge; not before a
    // two-level merge, where its early CTAs measured slower (32K tokens in
    // one layer: 16.0 vs 15.3 us per launch)
    if (NS <= kFan) pdl_trigger();

    // ---------------------------------------------------- warp finalisation
#pragma unroll
    for (int e = 0; e < 2; ++e) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], o);
        z_run[e] += __shfl_xor_sync(0xffffffffu, z_run[e], o);
      }
    }
    // NaN scores never raise the running maximum, so the merge would treat
    // such a warp as empty; its sums still carry the NaN: report it
    if (!(isfinite(l_run[0]) && isfinite(l_run[1]) && isfinite(z_run[0]) && isfinite(z_run[1])))
      atomicOr(&g_decode_nonfinite, 1u);
    __syncthreads();   // all warps done with their rings and the query slices
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
        const float inv = kKeyUnscale / code_factor<VB>(j);   // value codes carry f * 2^-24
#pragma unroll
        for (int e = 0; e < 2; ++e)
          mO[(warp * kHeads + 2 * t4 + e) * D + d] = fmaf(acc[mi][2 * hh + e], inv, z_run[e]);
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

    // ------------------------------------------------- CTA merge of the warps
    const int gqa = p.gqa;
    const bool xchg_mode = XCHG && p.x_signal != nullptr;
    const bool partial_mode = p.out_ml != nullptr || xchg_mode;
    const int64_t x_rows = (int64_t)p.n_layers * p.batch * p.HQ;
    const int64_t pstride = kHeads * (D + 2);
    const int x_e = xchg_mode ? s_xe : 0;
    auto emit = [&](int h, int d, float4 o, float M, float L) {
      const int64_t row = (int64_t)b * p.HQ + kvh * gqa + h;
      if (!(isfinite(o.x) && isfinite(o.y) && isfinite(o.z) && isfinite(o.w) && isfinite(L)))
        atomicOr(&g_decode_nonfinite, 1u);   // an fp16 operand left its range
      if (partial_mode) {
        const int64_t prow = (int64_t)layer * p.batch * p.HQ + row;
        if (xchg_mode) {
          // every rank's receive area, this rank's slot of the step's half:
          // each 8-byte word is (value, epoch), written whole, so the
          // receiver validates every word by its tag and nothing here waits
          // for the stores to land (no fence, no flag)
          const uint32_t e = (uint32_t)x_e;
          const int64_t lslot = x_rows * (2 + D) * 2;   // 32-bit words per (half, source)
          // owner mode: only the rank that merges this row receives it
          const int r_lo = p.x_owner ? (int)(prow % p.x_world) : 0;
          const int r_hi = p.x_owner ? r_lo + 1 : p.x_world;
          for (int r = r_lo; r < r_hi; ++r) {
            uint32_t* base = reinterpret_cast<uint32_t*>(p.x_signal[r]) + kLLWords +
                             ((int64_t)(x_e & 1) * p.x_world + p.x_rank) * lslot + prow * (2 + D) * 2;
            st_volatile_v4(base + 2 * (2 + d), __float_as_uint(o.x), e, __float_as_uint(o.y), e);
            st_volatile_v4(base + 2 * (2 + d + 2), __float_as_uint(o.z), e, __float_as_uint(o.w), e);
            if (d == 0) st_volatile_v4(base, __float_as_uint(M), e, __float_as_uint(L), e);
          }
        } else {
          *reinterpret_cast<float4*>(p.out_o + prow * D + d) = o;
          if (d == 0) { p.out_ml[2 * prow] = M; p.out_ml[2 * prow + 1] = L; }
        }
      } else {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const float4 r = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        if (p.out_f32) {
          *reinterpret_cast<float4*>(static_cast<float*>(Lp.out) + row * D + d) = r;
        } else {
          uint2 w;
          w.x = (uint32_t)f32_to_bf16_bits(r.x) | ((uint32_t)f32_to_bf16_bits(r.y) << 16);
          w.y = (uint32_t)f32_to_bf16_bits(r.z) | ((uint32_t)f32_to_bf16_bits(r.w) << 16);
          *reinterpret_cast<uint2*>(static_cast<uint16_t*>(Lp.out) + row * D + d) = w;
        }
      }
    };
    const bool clustered = NS > 1 && p.cluster > 1;
    float* cpart = reinterpret_cast<float*>(smem + C::CPART_OFF);
    float* my_part = NS > 1 ? (clustered ? cpart : p.part1 + ((int64_t)unit * NS + sp) * pstride) : nullptr;
    for (int idx = threadIdx.x; idx < gqa * (D / 4); idx += blockDim.x) {
      const int h = idx / (D / 4), d = 4 * (idx % (D / 4));
      float M = NEG_INF;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mM[w * kHeads + h]);
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      float l = 0.f;
      if (M != NEG_INF) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const float mw = mM[w * kHeads + h];
          const float wt = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
          const float4 ow = *reinterpret_cast<const float4*>(mO + (w * kHeads + h) * D + d);
          o.x = fmaf(wt, ow.x, o.x); o.y = fmaf(wt, ow.y, o.y);
          o.z = fmaf(wt, ow.z, o.z); o.w = fmaf(wt, ow.w, o.w);
          l = fmaf(wt, mL[w * kHeads + h], l);
        }
      }
      if (NS == 1) {
        emit(h, d, o, M, l);
      } else {
        *reinterpret_cast<float4*>(my_part + 2 * kHeads + h * D + d) = o;
        if (d == 0) { my_part[h] = M; my_part[kHeads + h] = l; }
      }
    }
    if (NS == 1) continue;

    // ---------------------------------------- two-level last-arriver merge
    // merge n (<= kFan) partials at src (stride pstride) into the partial
    // at dst, or into the final output when dst is null.  One warp per
    // head, lane = 4 consecutive d; every load of a head is issued before
    // the first use, so a merge costs one L2 round trip per head rather
    // than one per partial.
    // The loads come from global memory (split partials, src) or, in a
    // cluster (from_cluster), from the shared memory of the cluster's CTAs:
    // partial s is CTA s's cpart.  The source is a compile-time choice so
    // the global merge keeps all its loads in flight before the first use.
    auto merge = [&](auto from_cluster, const float* src, int n, float* dst, int h0, int h_step) {
      constexpr bool DSM = decltype(from_cluster)::value;
      for (int h = h0; h < gqa; h += h_step) {
        const int d = 4 * lane;
        const bool dl = d < D;
        float ms[kFan], ls[kFan];
        float4 vs[kFan];
#pragma unroll
        for (int s = 0; s < kFan; ++s) {
          const bool ok = s < n;
          if constexpr (DSM) {
            const uint32_t rs = ok ? dsmem_map(smem_u32(cpart), s) : 0u;
            ms[s] = ok ? dsmem_f32(rs + 4 * h) : NEG_INF;
            ls[s] = ok ? dsmem_f32(rs + 4 * (kHeads + h)) : 0.f;
            vs[s] = (ok && dl) ? dsmem_f32x4(rs + 4 * (2 * kHeads + h * D + d)) : make_float4(0.f, 0.f, 0.f, 0.f);
          } else {
            ms[s] = ok ? __ldcg(src + s * pstride + h) : NEG_INF;
            ls[s] = ok ? __ldcg(src + s * pstride + kHeads + h) : 0.f;
            vs[s] = (ok && dl) ? __ldcg(reinterpret_cast<const float4*>(src + s * pstride + 2 * kHeads + h * D + d))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        float M = NEG_INF;
#pragma unroll
        for (int s = 0; s < kFan; ++s) M = fmaxf(M, ms[s]);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
#pragma unroll
        for (int s = 0; s < kFan; ++s) {
          const float wt = (ms[s] == NEG_INF) ? 0.f : fast_exp2(ms[s] - M);
          o.x = fmaf(wt, vs[s].x, o.x); o.y = fmaf(wt, vs[s].y, o.y);
          o.z = fmaf(wt, vs[s].z, o.z); o.w = fmaf(wt, vs[s].w, o.w);
          L = fmaf(wt, ls[s], L);
        }
        if (M == NEG_INF) { o = make_float4(0.f, 0.f, 0.f, 0.f); L = 0.f; }
        if (dl) {
          if (dst) {
            *reinterpret_cast<float4*>(dst + 2 * kHeads + h * D + d) = o;
            if (d == 0) { dst[h] = M; dst[kHeads + h] = L; }
          } else {
            emit(h, d, o, M, L);
          }
        }
      }
    };
    if (clustered) {
      // Cluster merge (the cluster is all NS splits of this unit): every
      // CTA's partial sits in its own shared memory; the heads are dealt
      // out over the cluster's CTAs and warps (head h to CTA h % NS), each
      // merged over distributed shared memory straight into the output, so
      // the merge and its output stores are spread over NS SMs.  The second
      // barrier keeps every CTA's shared memory alive until all have read it.
      cluster_sync_all();
      merge(std::true_type{}, nullptr, NS, nullptr, (int)cluster_rank() + NS * warp, NS * kWarps);
      cluster_sync_all();
      continue;
    }
    const int G1 = p.groups1;
    const int grp1 = sp / kFan;
    const int n1 = min(kFan, NS - grp1 * kFan);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_flag = (atomicAdd(p.cnt1 + (int64_t)unit * G1 + grp1, 1) == n1 - 1);
    __syncthreads();
    if (!s_flag) continue;
    __threadfence();
    const float* src1 = p.part1 + ((int64_t)unit * NS + grp1 * kFan) * pstride;
    if (G1 == 1) {
      merge(std::false_type{}, src1, n1, nullptr, warp, kWarps);
      if (threadIdx.x == 0) p.cnt1[(int64_t)unit * G1 + grp1] = 0;
      continue;
    }
    merge(std::false_type{}, src1, n1, p.part2 + ((int64_t)unit * G1 + grp1) * pstride, warp, kWarps);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      p.cnt1[(int64_t)unit * G1 + grp1] = 0;
      s_flag = (atomicAdd(p.cnt2 + unit, 1) == G1 - 1);
    }
    __syncthreads();
    if (!s_flag) continue;
    __threadfence();
    merge(std::false_type{}, p.part2 + (int64_t)unit * G1 * pstride, G1, nullptr, warp, kWarps);
    if (threadIdx.x == 0) p.cnt2[unit] = 0;
  }
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
  int num_splits = 1, chunks_per_split = 1, items = 1, grid = 1, groups1 = 1, cluster = 1;
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

// Choose the split count with a small cost model: time ~ waves x (chunks per
// warp + fixed per-item cost) + merge cost; the persistent grid strides
// over the items, so a wave is `slots` = SMs x resident CTAs per SM.
static Plan make_plan(const kvr_decode_args* a, int tok_begin, int tok_end, int ctas_per_sm) {
  Plan pl;
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  const int nchunks = std::max(1, (tok_end - tok_begin + kChunk - 1) / kChunk);
  const int64_t slots = (int64_t)device_sms(a->num_sms) * std::max(1, ctas_per_sm);
  int ns;
  if (a->split_tokens > 0) {
    const int cps = std::max(1, (a->split_tokens + kChunk - 1) / kChunk);
    ns = (nchunks + cps - 1) / cps;
  } else {
    double best = 1e30;
    ns = 1;
    const int ns_max = std::min(kMaxSplits, std::max(1, nchunks / 2));
    for (int cand = 1; cand <= ns_max; ++cand) {
      const int cps = (nchunks + cand - 1) / cand;
      const int real = (nchunks + cps - 1) / cps;
      if (real != cand) continue;
      const int64_t items = units * cand;
      const int64_t waves = (items + slots - 1) / slots;
      const double per_item = (double)cps / kWarps + 1.5;
      // merge cost, in units of one chunk per warp (about 1 us when a launch
      // is latency-bound).  A plan that fits in one wave merges up to kFan
      // splits in a thread-block cluster (about 2) and more splits in two
      // global levels whose cost grows with the second level's fan-in
      // (5 + groups/4); both fitted to single-layer launches on B200
      // (e.g. 4K tokens: 16 splits 8.8 us vs 64 splits 11.1 us; 32K: 128
      // splits 15.1 us vs 256 splits 16.8 us).  Plans of several waves
      // overlap the merge with other items' work.
      double merge = cand > 1 ? 1.0 + (cand > kFan ? 1.0 : 0.0) : 0.0;
      if (cand > 1 && items <= slots)
        merge = cand <= kFan ? 2.0 : 5.0 + (double)((cand + kFan - 1) / kFan) / 4.0;
      const double t = waves * per_item + merge;
      if (t < best - 1e-9) { best = t; ns = cand; }
    }
  }
  ns = std::min(ns, kMaxSplits);
  const int cps = (nchunks + ns - 1) / ns;
  ns = (nchunks + cps - 1) / cps;
  pl.num_splits = ns;
  pl.chunks_per_split = cps;
  pl.items = (int)std::min<int64_t>(units * ns, 0x7fffffff);
  pl.grid = (int)std::min<int64_t>(pl.items, slots);
  pl.groups1 = (ns + kFan - 1) / kFan;
  pl.counters = (size_t)units * (pl.groups1 + 1);
  const size_t pstride = (size_t)kHeads * (a->head_dim + 2);
  pl.part_bytes = ns > 1 ? (size_t)units * (ns + (pl.groups1 > 1 ? pl.groups1 : 0)) * pstride * 4 : 0;
  return pl;
}

// make_plan memoised per host thread: a decode loop re-plans the same shape
// every step (the cost model scans up to kMaxSplits candidates).
static Plan cached_plan(const kvr_decode_args* a, int tb, int te, int occ) {
  struct Entry {
    int key[10];
    Plan plan;
  };
  static thread_local Entry cache[8];
  static thread_local int next = 0;
  const int key[10] = {a->n_layers, a->batch, a->kv_heads, a->head_dim, tb, te, a->split_tokens,
                       device_sms(a->num_sms), occ, 1};
  for (auto& e : cache)
    if (std::equal(key, key + 10, e.key)) return e.plan;
  Entry& e = cache[next];
  next = (next + 1) % 8;
  std::copy(key, key + 10, e.key);
  e.plan = make_plan(a, tb, te, occ);
  return e.plan;
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
  if (a->out_dtype != 0 && a->out_dtype != 1) return KVR_ERR_INVALID_ARGUMENT;
  // key group: a power of two, at least one 16-token mma tile
  if (a->group_size < 16 || (a->group_size & (a->group_size - 1))) return KVR_ERR_UNSUPPORTED;
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
        (L.key_residual && !aligned16(L.key_residual)) || !aligned16(L.query) || !aligned16(L.out) ||
        (L.key_scale_pairs && !aligned16(L.key_scale_pairs)))
      return KVR_ERR_MISALIGNED;
  }
  return KVR_OK;
}

template <int MAXL>
static void fill_params(Params<MAXL>& p, const kvr_decode_args* a, const Plan& pl, int tb, int te) {
  for (int l = 0; l < a->n_layers; ++l) {
    const kvr_layer_ptrs& L = a->layers[l];
    p.L[l] = LayerPtrs{L.key_payload, L.key_scale, L.key_offset, L.key_residual, L.value_payload,
                       L.value_scale, L.value_offset, L.query, L.out, L.key_scale_pairs};
  }
  p.n_layers = a->n_layers;
  p.BH = a->batch * a->kv_heads;
  p.HQ = a->q_heads;
  p.HKV = a->kv_heads;
  p.gqa = a->q_heads / a->kv_heads;
  p.batch = a->batch;
  p.S = a->seq_len;
  p.P = a->prefix_len;
  p.G = a->group_size;
  int lg = 0;
  while ((1 << lg) < a->group_size) ++lg;
  p.log2G = lg;
  p.tok_begin = tb;
  p.tok_end = te;
  p.num_splits = pl.num_splits;
  p.chunks_per_split = pl.chunks_per_split;
  p.items = pl.items;
  p.groups1 = pl.groups1;
  p.kp_bh = a->key_payload_bh_stride;
  p.km_bh = a->key_meta_bh_stride;
  p.kr_bh = a->key_residual_bh_stride;
  p.vp_bh = a->value_payload_bh_stride;
  p.vm_bh = a->value_meta_bh_stride;
  bool staged = a->value_meta_bh_stride % 8 == 0;
  for (int l = 0; l < a->n_layers; ++l)
    staged = staged && aligned16(a->layers[l].value_scale) && aligned16(a->layers[l].value_offset);
  p.vm_staged = staged ? 1 : 0;
  p.score_scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)a->head_dim));
  p.out_f32 = a->out_dtype == 1;
  const int64_t units = (int64_t)a->n_layers * a->batch * a->kv_heads;
  const int64_t pstride = (int64_t)kHeads * (a->head_dim + 2);
  p.part1 = pl.num_splits > 1 ? static_cast<float*>(a->workspace) : nullptr;
  p.part2 = (pl.num_splits > 1 && pl.groups1 > 1) ? p.part1 + units * pl.num_splits * pstride : nullptr;
  p.cnt1 = a->counters;
  p.cnt2 = a->counters ? a->counters + units * pl.groups1 : nullptr;
  p.out_ml = nullptr;
  p.out_o = nullptr;
  p.dev_len = nullptr;
  p.res_cap = a->seq_len - a->prefix_len;
  p.cluster = pl.cluster;
  p.q_shared = a->query_host_mapped ? 1 : 0;
  p.app_k = nullptr;
  p.app_v = nullptr;
  p.x_signal = nullptr;
  p.x_epoch = nullptr;
  p.x_world = 0;
  p.x_rank = 0;
  p.x_owner = 0;
}

// Per-device, per-instantiation set-up: dynamic shared memory limit and
// resident CTAs per SM (a benign race sets the same values).
template <int D, int KB, int VB, int MAXL, bool XCHG = false>
static int prepare(int* ctas_per_sm) {
  using C = Cfg<D, KB, VB>;
  auto kern = decode_kernel<D, KB, VB, MAXL, XCHG>;
  static int occ[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  dev &= 63;
  if (occ[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    // ask for the full shared-memory carveout so the resident-CTA count the
    // persistent grid is sized for is what the SM actually hosts
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    // clusters of up to 16 CTAs (the cluster merge); refused on parts without them
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      (void)cudaGetLastError();
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kWarps * 32, C::SMEM);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    occ[dev] = std::max(1, n);
  }
  *ctas_per_sm = occ[dev];
  return KVR_OK;
}

// Clusters of `cl` CTAs that can be resident at once on this device (0 when
// the size is unsupported), per device and size.
template <int D, int KB, int VB, int MAXL, bool XCHG = false>
static int active_clusters(int cl) {
  static int cache[64][17];
  static bool init[64][17];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  dev &= 63;
  if (cl < 2 || cl > 16) return 0;
  if (!init[dev][cl]) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(cl);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = Cfg<D, KB, VB>::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, decode_kernel<D, KB, VB, MAXL, XCHG>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    cache[dev][cl] = n;
    init[dev][cl] = true;
  }
  return cache[dev][cl];
}

// Cluster size for a plan: all splits of a unit in one cluster (at most
// kFan of them, so the partials are merged in the same order as the global
// single-level merge and the output is bit-identical to it), only when every
// CTA takes exactly one item and the device holds every cluster at once.
// With more splits, clusters of kFan plus a global level measured slower on
// B200 than two global levels (uneven cluster placement over the GPCs and a
// costlier launch), so those plans keep the global merge.
template <int D, int KB, int VB, int MAXL, bool XCHG = false>
static int cluster_for(const Plan& pl) {
  const int ns = pl.num_splits;
  if (ns < 2 || ns > kFan || pl.items > pl.grid) return 1;
  const int n = active_clusters<D, KB, VB, MAXL, XCHG>(ns);
  return (n > 0 && pl.items / ns <= n) ? ns : 1;
}

template <int D, int KB, int VB, int MAXL, bool XCHG = false>
static void launch(const Params<MAXL>& p, const Plan& pl, cudaStream_t s) {
  (void)pdl_launch(decode_kernel<D, KB, VB, MAXL, XCHG>, dim3(pl.grid), dim3(kWarps * 32), Cfg<D, KB, VB>::SMEM, s,
                   pl.cluster, p);
}

template <int MAXL>
static void set_exchange(Params<MAXL>& p, const kvr_exchange_args* x) {
  if (!x) return;
  p.x_signal = x->signal;
  p.x_epoch = x->epoch;
  p.x_world = x->world;
  p.x_rank = x->rank;
  p.x_owner = x->mode == 1 ? 1 : 0;
}

template <int D, int KB, int VB>
static int run_t(const kvr_decode_args* a, int tb, int te, float* out_ml, float* out_o, cudaStream_t s,
                 Plan* plan_only, const int* dev_len, int res_cap, const uint16_t* app_k,
                 const uint16_t* app_v, const kvr_exchange_args* x) {
  using C = Cfg<D, KB, VB>;
  int occ = 3;
  // the fused exchange has one instantiation, over the multi-layer parameter block
  const int dev_st = x                     ? prepare<D, KB, VB, KVR_MAX_LAYERS, true>(&occ)
                     : (a->n_layers == 1) ? prepare<D, KB, VB, 1>(&occ)
                                          : prepare<D, KB, VB, KVR_MAX_LAYERS>(&occ);
  if (dev_st != KVR_OK) {
    // no usable device: plan with a shared-memory-bound estimate; argument
    // errors below still take precedence over the device error
    occ = std::max(1, std::min(C::MIN_CTAS, (228 * 1024) / (C::SMEM + 1024)));
  }
  Plan pl = cached_plan(a, tb, te, occ);
  if (plan_only) {
    if (dev_st == KVR_OK)
      pl.cluster = x                     ? cluster_for<D, KB, VB, KVR_MAX_LAYERS, true>(pl)
                   : (a->n_layers == 1) ? cluster_for<D, KB, VB, 1>(pl)
                                        : cluster_for<D, KB, VB, KVR_MAX_LAYERS>(pl);
    *plan_only = pl;
    return KVR_OK;
  }
  if (pl.num_splits > 1) {
    if (!a->workspace || a->workspace_bytes < pl.part_bytes || !a->counters) return KVR_ERR_WORKSPACE;
    if (!aligned16(a->workspace)) return KVR_ERR_MISALIGNED;
  }
  if (dev_st != KVR_OK) return dev_st;
  if (a->n_layers == 1 && !x) {
    pl.cluster = cluster_for<D, KB, VB, 1>(pl);
    Params<1> p;
    fill_params(p, a, pl, tb, te);
    p.out_ml = out_ml; p.out_o = out_o;
    if (dev_len) { p.dev_len = const_cast<int*>(dev_len); p.res_cap = res_cap; }
    p.app_k = app_k; p.app_v = app_v;
    launch<D, KB, VB, 1>(p, pl, s);
  } else if (x) {
    pl.cluster = cluster_for<D, KB, VB, KVR_MAX_LAYERS, true>(pl);
    Params<KVR_MAX_LAYERS> p;
    fill_params(p, a, pl, tb, te);
    set_exchange(p, x);
    launch<D, KB, VB, KVR_MAX_LAYERS, true>(p, pl, s);
  } else {
    pl.cluster = cluster_for<D, KB, VB, KVR_MAX_LAYERS>(pl);
    Params<KVR_MAX_LAYERS> p;
    fill_params(p, a, pl, tb, te);
    p.out_ml = out_ml; p.out_o = out_o;
    if (dev_len) { p.dev_len = const_cast<int*>(dev_len); p.res_cap = res_cap; }
    p.app_k = app_k; p.app_v = app_v;
    launch<D, KB, VB, KVR_MAX_LAYERS>(p, pl, s);
  }
  return check_launch();
}

static int run(const kvr_decode_args* a, int tb, int te, float* out_ml, float* out_o, cudaStream_t s,
               Plan* plan_only = nullptr, const int* dev_len = nullptr, int res_cap = 0,
               const uint16_t* app_k = nullptr, const uint16_t* app_v = nullptr,
               const kvr_exchange_args* x = nullptr) {
  int st = validate(a);
  if (st != KVR_OK) return st;
  if (tb < 0 || te > a->seq_len || tb >= te || tb % kChunk) return KVR_ERR_INVALID_ARGUMENT;
#define KVR_CASE(D_, KB_, VB_)                                                              \
  if (a->head_dim == D_ && a->key_bits == KB_ && a->value_bits == VB_)                      \
    return run_t<D_, KB_, VB_>(a, tb, te, out_ml, out_o, s, plan_only, dev_len, res_cap, app_k, app_v, x);
  KVR_CASE(128, 4, 4) KVR_CASE(128, 8, 4) KVR_CASE(128, 4, 8) KVR_CASE(128, 8, 8)
  KVR_CASE(128, 2, 2) KVR_CASE(128, 2, 4) KVR_CASE(128, 4, 2) KVR_CASE(128, 8, 2) KVR_CASE(128, 2, 8)
  KVR_CASE(64, 4, 4) KVR_CASE(64, 8, 4) KVR_CASE(64, 4, 8) KVR_CASE(64, 8, 8) KVR_CASE(64, 2, 4)
  KVR_CASE(64, 2, 8)
#undef KVR_CASE
  return KVR_ERR_UNSUPPORTED;
}

}  // namespace dec
}  // namespace kvr

using namespace kvr;

extern "C" int kvr_decode_plan(const kvr_decode_args* a, int* num_splits, size_t* workspace_bytes,
                               size_t* counter_count) {
  if (!a) return KVR_ERR_INVALID_ARGUMENT;
  dec::Plan pl;
  int st = dec::run(a, 0, a->seq_len, nullptr, nullptr, nullptr, &pl);
  if (st != KVR_OK) return st;
  if (num_splits) *num_splits = pl.num_splits;
  if (workspace_bytes) *workspace_bytes = pl.part_bytes;
  if (counter_count) *counter_count = pl.counters;
  return KVR_OK;
}

extern "C" int kvr_decode_cluster(const kvr_decode_args* a, int* cluster) {
  if (!a || !cluster) return KVR_ERR_INVALID_ARGUMENT;
  dec::Plan pl;
  int st = dec::run(a, 0, a->seq_len, nullptr, nullptr, nullptr, &pl);
  if (st != KVR_OK) return st;
  *cluster = pl.cluster;
  return KVR_OK;
}

extern "C" int kvr_decode_attention(const kvr_decode_args* a, kvr_stream_t stream) {
  if (!a) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, 0, a->seq_len, nullptr, nullptr, as_stream(stream));
}

extern "C" int kvr_decode_attention_lengths(const kvr_decode_args* a, const int* lengths, int residual_capacity,
                                            kvr_stream_t stream) {
  if (!a || !lengths || residual_capacity < 0) return KVR_ERR_INVALID_ARGUMENT;
  if (a->seq_len - a->prefix_len > residual_capacity) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, 0, a->seq_len, nullptr, nullptr, as_stream(stream), nullptr, lengths, residual_capacity);
}

extern "C" int kvr_decode_step(const kvr_decode_args* a, const uint16_t* k_new, const uint16_t* v_new, int* lengths,
                               int residual_capacity, kvr_stream_t stream) {
  if (!a || !lengths || !k_new || !v_new || residual_capacity < 0 || a->n_layers != 1)
    return KVR_ERR_INVALID_ARGUMENT;
  if (a->seq_len - a->prefix_len > residual_capacity) return KVR_ERR_INVALID_ARGUMENT;
  if (!aligned16(k_new) || !aligned16(v_new)) return KVR_ERR_MISALIGNED;
  return dec::run(a, 0, a->seq_len, nullptr, nullptr, as_stream(stream), nullptr, lengths, residual_capacity, k_new,
                  v_new);
}

extern "C" int kvr_decode_partial(const kvr_decode_args* a, int token_begin, int token_end, float* part_ml,
                                  float* part_o, kvr_stream_t stream) {
  if (!a || !part_ml || !part_o) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, token_begin, token_end, part_ml, part_o, as_stream(stream));
}

extern "C" int kvr_decode_partial_exchange(const kvr_decode_args* a, int token_begin, int token_end,
                                           const kvr_exchange_args* x, kvr_stream_t stream) {
  if (!a || !x || x->world < 1 || x->world > 8 || x->rank < 0 || x->rank >= x->world || !x->signal || !x->epoch)
    return KVR_ERR_INVALID_ARGUMENT;
  if (x->rows != a->n_layers * a->batch * a->q_heads || x->head_dim != a->head_dim) return KVR_ERR_INVALID_ARGUMENT;
  return dec::run(a, token_begin, token_end, nullptr, nullptr, as_stream(stream), nullptr, nullptr, 0, nullptr,
                  nullptr, x);
}

// ---------------------------------------------------------------------------
// Key scales as fp16 pairs in the decode kernel's register order
// (kvr_layer_ptrs.key_scale_pairs).  Word w = t4 * D/8 + r of a group holds
// the scales of the two channels key register r of lane slice t4 covers,
// dbase + key_dlocal(r, 0) and dbase + key_dlocal(r, 1) (dbase = t4 * D/4),
// rounded to fp16 exactly as the decode kernel rounds them (cvt.rn from the
// bf16 value), so a decode reading the table equals one converting per chunk.
namespace kvr {
namespace dec {
template <int D, int KB>
__global__ void __launch_bounds__(256) scale_pairs_kernel(const kvr_scale_pairs_args a) {
  constexpr int W = D / 2;   // 32-bit words per group
  const int64_t n = (int64_t)a.bh * a.groups * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % W);
    const int64_t rest = i / W;
    const int64_t grp = a.group0 + rest % a.groups;
    const int64_t bh = rest / a.groups;
    const int t4 = w / (D / 8), r = w % (D / 8);
    const int d0 = t4 * (D / 4) + key_dlocal<KB>(r, 0), d1 = t4 * (D / 4) + key_dlocal<KB>(r, 1);
    const uint16_t* s = a.scale + bh * a.scale_bh_stride + grp * D;
    const uint32_t word = pack_half2(bf16_bits_to_f32(s[d0]), bf16_bits_to_f32(s[d1]));
    *reinterpret_cast<uint32_t*>(a.pairs + bh * a.pairs_bh_stride + grp * D + 2 * w) = word;
  }
}
}  // namespace dec
}  // namespace kvr

extern "C" int kvr_key_scale_pairs(const kvr_scale_pairs_args* a, kvr_stream_t stream) {
  if (!a || !a->scale || !a->pairs || a->bh < 0 || a->groups < 0 || a->group0 < 0) return KVR_ERR_INVALID_ARGUMENT;
  if (a->head_dim != 64 && a->head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (a->key_bits != 2 && a->key_bits != 4 && a->key_bits != 8) return KVR_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a->pairs) & 3u) || (a->pairs_bh_stride & 1)) return KVR_ERR_MISALIGNED;
  const int64_t n = (int64_t)a->bh * a->groups * (a->head_dim / 2);
  if (n == 0) return KVR_OK;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  cudaStream_t s = as_stream(stream);
#define KVR_PAIRS(D_, KB_)                                                        \
  if (a->head_dim == D_ && a->key_bits == KB_) {                                  \
    dec::scale_pairs_kernel<D_, KB_><<<blocks, 256, 0, s>>>(*a);                   \
    return check_launch();                                                        \
  }
  KVR_PAIRS(128, 2) KVR_PAIRS(128, 4) KVR_PAIRS(128, 8) KVR_PAIRS(64, 2) KVR_PAIRS(64, 4) KVR_PAIRS(64, 8)
#undef KVR_PAIRS
  return KVR_ERR_UNSUPPORTED;
}

extern "C" int kvr_decode_nonfinite(int* flag, int clear) {
  if (!flag) return KVR_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaDeviceSynchronize();
  unsigned int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, dec::g_decode_nonfinite, sizeof(v));
  if (e == cudaSuccess && clear && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(dec::g_decode_nonfinite, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  *flag = v ? 1 : 0;
  return KVR_OK;
}

// ---------------------------------------------------------------------------
// Decode attention for callers that cannot allocate device memory.
//
// Some callers of this library have no device allocator to hand: an FFI host
// (Go, Java, a C engine) that owns no CUDA memory pool, a real-time serving
// loop that must not call cudaMalloc (it can synchronize the device and stall
// every stream), or code running under a fixed memory budget.  They cannot
// provide the split-partial workspace kvr_decode_attention asks for, so this
// entry point keeps that scratch in a fixed array compiled into the library.
//
// The array is file-scope device memory: every GPU that loads the library
// holds it until the process exits.  Host code cannot use the array's name
// as a device address; its address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on
// that device -- so make the first call on each device before any stream
// capture.  All calls share the array and it keeps the last call's contents:
// each call clears the split counters it uses, and two calls that overlap on
// the GPU (different streams, or concurrent graph launches) race.
namespace kvr {
namespace dec {
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;   // 4 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Device address of the array, per device ordinal.  Host threads making
// their first call on a device at the same time may both look it up; they
// store the same value, and the atomic makes that race well defined.
static std::atomic<void*> g_noalloc_base[64];

static int noalloc_base(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  if (dev < 0 || dev >= 64) return KVR_ERR_UNSUPPORTED;
  void* p = g_noalloc_base[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
    g_noalloc_base[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return KVR_OK;
}
}  // namespace dec
}  // namespace kvr

extern "C" int kvr_decode_attention_noalloc(const kvr_decode_args* a, kvr_stream_t stream) {
  if (!a) return KVR_ERR_INVALID_ARGUMENT;
  dec::Plan pl;
  int st = dec::run(a, 0, a->seq_len, nullptr, nullptr, nullptr, &pl);   // validates, plans
  if (st != KVR_OK) return st;
  const size_t counter_bytes = (pl.counters * sizeof(int) + 255) / 256 * 256;
  if (counter_bytes + pl.part_bytes > dec::kNoAllocScratchBytes) return KVR_ERR_WORKSPACE;
  void* base = nullptr;
  st = dec::noalloc_base(&base);
  if (st != KVR_OK) return st;
  kvr_decode_args b = *a;
  b.counters = static_cast<int*>(base);
  b.workspace = static_cast<unsigned char*>(base) + counter_bytes;
  b.workspace_bytes = dec::kNoAllocScratchBytes - counter_bytes;
  if (pl.num_splits > 1) {
    // the array keeps the previous call's contents: counters must start at zero
    cudaError_t e = cudaMemsetAsync(b.counters, 0, pl.counters * sizeof(int), as_stream(stream));
    if (e != cudaSuccess) { set_last_cuda_error(e); return KVR_ERR_CUDA; }
  }
  return dec::run(&b, 0, a->seq_len, nullptr, nullptr, as_stream(stream));
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
