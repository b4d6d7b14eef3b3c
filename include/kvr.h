/*
 * kvr.h -- C ABI of the B200-native packed draft-KV hot path.
 *
 * Every entry point takes plain device pointers, element counts and strides,
 * enqueues its work on the given CUDA stream (a cudaStream_t passed as void*,
 * NULL = legacy default stream) and returns an int status (KVR_OK = 0).  No
 * entry point allocates device memory; callers pass outputs and workspaces.
 *
 * Tensor layouts follow kv_reduce/packed_kv_cache.py of the reference:
 *   key payload    uint8  [B, H, P, D*kb/8]   codes LSB-first within bytes
 *   key scale/off  bf16   [B, H, P/G, D]      (reference shape [B,H,P/G,1,D])
 *   key residual   bf16   [B, H, S-P, D]      the BF16 window after the prefix
 *   value payload  uint8  [B, H, S, D*vb/8]
 *   value scale/off bf16  [B, H, S]           (reference shape [B,H,S,1])
 * where P = floor(max(0, S-R)/G)*G  (packed_kv_cache.py:15-19).
 * Each (b,h) slab is addressed through an explicit "bh stride", so the
 * reference's contiguous slabs (stride = P*D*kb/8 ...) and a preallocated
 * capacity layout (stride = capacity*...) are both accepted.
 */
#ifndef KVR_H_
#define KVR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* kvr_stream_t;

enum kvr_status {
  KVR_OK = 0,
  KVR_ERR_INVALID_ARGUMENT = 1,   /* bad size, bit width, null pointer ... */
  KVR_ERR_UNSUPPORTED = 2,        /* valid for the reference, not built here */
  KVR_ERR_MISALIGNED = 3,         /* pointer/stride breaks a 16-byte rule */
  KVR_ERR_CUDA = 4,               /* a CUDA runtime call failed */
  KVR_ERR_CAPACITY = 5,           /* streaming cache would overflow */
  KVR_ERR_WORKSPACE = 6           /* workspace smaller than kvr_decode_plan asked */
};

#define KVR_MAX_LAYERS 32

/* Library version (major*10000 + minor*100 + patch). */
int kvr_version(void);
/* Human-readable text for a kvr_status value. */
const char* kvr_status_string(int status);
/* Last CUDA error text seen by the library on this host thread ("" if none). */
const char* kvr_last_error(void);
/* *mapped = 1 when p points into page-locked host memory that the current
 * device reads and writes at the same address (unified addressing), so a
 * kernel may take it as a device pointer, else 0.  No reference
 * counterpart: the host-buffer decode step uses it to let the decode write
 * its outputs straight into pinned host memory.                            */
int kvr_host_mapped(const void* p, int* mapped);

/* ---------------------------------------------------------------- packing
 * Replaces pack_unsigned (packed_kv_cache.py:28-63): n codes (uint8, each
 * < 2^bits) -> ceil(n*bits/8) bytes, value i at bit i*bits, LSB first.
 * bits in [1, 8].  Codes >= 2^bits are masked (the reference raises on the
 * host; the Python layer keeps that check).                                */
int kvr_pack_unsigned(const uint8_t* codes, int64_t n, int bits,
                      uint8_t* payload, kvr_stream_t stream);

/* Replaces unpack_unsigned (packed_kv_cache.py:66-94). */
int kvr_unpack_unsigned(const uint8_t* payload, int64_t n, int bits,
                        uint8_t* codes, kvr_stream_t stream);

/* ------------------------------------------------------- quantize + pack
 * Values, per-token affine: replaces pack_per_token_affine
 * (packed_kv_cache.py:159-192).  x: bf16 rows of D elements; row r of
 * (b,h) slab at x + bh*x_bh_stride + r*x_row_stride (elements).
 * Writes rows [row0, row0+rows) of payload/scale/offset for every (b,h):
 *   payload + bh*payload_bh_stride + (row0+r)*D*bits/8  (bytes)
 *   scale/offset + bh*meta_bh_stride + row0 + r        (elements)
 * bits in [2, 8].  When D*bits % 8 != 0 the reference's flat bitstream
 * crosses rows: then the payload is that flat stream of [bh, rows, D]
 * codes (payload_bh_stride unused), row0 must be 0 and `codes_scratch`
 * (bh*rows*D bytes) carries the codes between the two passes.             */
typedef struct {
  const uint16_t* x; int64_t x_bh_stride; int64_t x_row_stride;
  uint8_t* payload; int64_t payload_bh_stride;
  uint16_t* scale; uint16_t* offset; int64_t meta_bh_stride;
  int bh;          /* number of (b,h) slabs = B*H */
  int rows;        /* tokens to quantize per slab */
  int row0;        /* first destination token row */
  int head_dim;    /* D */
  int bits;
  uint8_t* codes_scratch;   /* only for the generic path, else NULL */
} kvr_token_quant_args;
int kvr_quantize_per_token(const kvr_token_quant_args* a, kvr_stream_t stream);

/* Keys, per-channel grouped affine over the token axis: replaces
 * pack_per_channel_grouped_affine (packed_kv_cache.py:195-253) for the
 * groups [group0, group0+groups) of every (b,h) slab.  Token t of a group
 * g is x row (g-group0)*G + t.  Payload row index = g*G + t.
 * scale/offset index = g*D + d (plus bh*meta_bh_stride).                  */
typedef struct {
  const uint16_t* x; int64_t x_bh_stride; int64_t x_row_stride;
  uint8_t* payload; int64_t payload_bh_stride;
  uint16_t* scale; uint16_t* offset; int64_t meta_bh_stride;
  int bh;
  int groups;      /* groups to quantize per slab */
  int group0;      /* first destination group */
  int group_size;  /* G */
  int head_dim;
  int bits;
  uint8_t* codes_scratch;   /* D*bits % 8 != 0 only; group0 must be 0 */
} kvr_group_quant_args;
int kvr_quantize_grouped(const kvr_group_quant_args* a, kvr_stream_t stream);

/* --------------------------------------------------------- dequantize
 * Replaces PackedKVComponent.unpack() (packed_kv_cache.py:126-149):
 * out = (code * scale + offset) in fp32 with separate roundings, then cast
 * to out_dtype (0 = bf16, 1 = fp32, 2 = fp16).  For keys the BF16 residual rows
 * [P, S) are copied after the dequantized prefix.                         */
typedef struct {
  const uint8_t* payload; int64_t payload_bh_stride;
  const uint16_t* scale; const uint16_t* offset; int64_t meta_bh_stride;
  const uint16_t* residual; int64_t residual_bh_stride;  /* keys only */
  void* out;       /* [bh, seq_len, D] contiguous */
  int out_dtype;   /* 0 bf16, 1 fp32, 2 fp16 */
  int bh;
  int seq_len;     /* S */
  int prefix_len;  /* P (keys) ; ignored for values */
  int group_size;  /* G (keys) ; 0 selects the per-token (value) layout */
  int head_dim;
  int bits;
} kvr_dequant_args;
int kvr_dequantize(const kvr_dequant_args* a, kvr_stream_t stream);

/* ------------------------------------------------------- streaming cache
 * One decode/draft step of PackedLayer.append (packed_review.py:23-31) on a
 * preallocated capacity layout: n new tokens per (b,h).  Keys go to the
 * BF16 residual rows [res_len, res_len+n); values are quantized per token
 * into rows [seq_len, seq_len+n) of the value payload/scale/offset.
 * Layout of the new tokens: k/v [bh, n, D] contiguous bf16.                */
typedef struct {
  const uint16_t* k; const uint16_t* v;
  uint16_t* key_residual; int64_t key_residual_bh_stride;
  uint8_t* value_payload; int64_t value_payload_bh_stride;
  uint16_t* value_scale; uint16_t* value_offset; int64_t value_meta_bh_stride;
  int bh, n, seq_len, res_len, res_capacity, seq_capacity, head_dim, value_bits;
} kvr_append_args;
int kvr_append(const kvr_append_args* a, kvr_stream_t stream);

/* PackedLayer.commit (packed_review.py:32-41): quantize the first
 * `groups` groups of the residual window into key groups
 * [prefix_len/G, prefix_len/G + groups) and move the remaining
 * res_len - groups*G residual rows to the front of `residual_out`
 * (a second buffer; the caller swaps buffers after the call).             */
typedef struct {
  const uint16_t* residual_in; uint16_t* residual_out; int64_t residual_bh_stride;
  uint8_t* key_payload; int64_t key_payload_bh_stride;
  uint16_t* key_scale; uint16_t* key_offset; int64_t key_meta_bh_stride;
  int bh, res_len, groups, prefix_len, prefix_capacity, group_size, head_dim, key_bits;
} kvr_flush_args;
int kvr_flush_groups(const kvr_flush_args* a, kvr_stream_t stream);

/* Lengths in device memory, for decode loops captured once in a CUDA graph
 * and replayed at growing lengths (no reference counterpart: the reference
 * passes lengths from the host on every call).  lengths is int[4]:
 * [0] sequence length, [1] quantized prefix length, [2] error flag,
 * [3] zero (scratch of the append's arrival count).
 * kvr_append_lengths: kvr_append with seq_len / res_len read from lengths
 *   at run time (a->seq_len, a->res_len ignored); an append past
 *   a->seq_capacity or a->res_capacity writes nothing and sets lengths[2];
 *   advance != 0: lengths[0] += a->n once the append is complete.
 * kvr_advance_lengths: lengths[0] += n unless the error flag is set.
 * kvr_set_lengths: lengths[0] = seq_len, lengths[1] = prefix_len.          */
int kvr_append_lengths(const kvr_append_args* a, int* lengths, int advance, kvr_stream_t stream);
int kvr_advance_lengths(int* lengths, int n, kvr_stream_t stream);
int kvr_set_lengths(int* lengths, int seq_len, int prefix_len, kvr_stream_t stream);

/* -------------------------------------------------------- decode attention
 * Replaces packed_kv_decode_attention (triton_packed_kv_attention.py:284-389)
 * and its three kernels (:27-131, :134-248, :251-281): one-token GQA decode
 * over the packed cache, split-K over tokens, online softmax in fp32, LSE
 * merge of the splits fused into the same launch.  Several layers of equal
 * geometry may share one launch (n_layers <= KVR_MAX_LAYERS).
 * query: [B, HQ, 1, D] bf16, out: [B, HQ, 1, D] bf16 or fp32, contiguous.
 * Supported: D in {64,128}; key/value bits in {2,4,8} (D=64 needs value
 * bits >= 4); G a multiple of 16 with G <= 128 or G == 16*k; HQ/HKV <= 8.
 * The caller passes a workspace of kvr_decode_plan() bytes for the split
 * partials (scratch, any contents) and `counters`, kvr_decode_plan() ints
 * that must be zero before the first launch; every completed launch leaves
 * them zero again, so one counter array can serve a stream's launches.     */
typedef struct {
  const uint8_t* key_payload;
  const uint16_t* key_scale;
  const uint16_t* key_offset;
  const uint16_t* key_residual;
  const uint8_t* value_payload;
  const uint16_t* value_scale;
  const uint16_t* value_offset;
  const uint16_t* query;
  void* out;            /* bf16 or fp32, see kvr_decode_args.out_dtype */
  /* Optional, NULL to leave it out: key_scale as fp16 pairs in the decode
   * kernel's register order, written from key_scale by kvr_key_scale_pairs
   * (same shape and strides as key_scale).  Given it, the decode reads these
   * pairs in place of the bf16 scales (the same number of bytes) instead of
   * converting every group's scales for each query head; the output is
   * bit-identical.  Zero-initialise the struct so the field is NULL when
   * unused.                                                                */
  const uint16_t* key_scale_pairs;
} kvr_layer_ptrs;

typedef struct {
  const kvr_layer_ptrs* layers;   /* host array of n_layers entries */
  int n_layers;
  int batch, q_heads, kv_heads, head_dim;
  int seq_len, prefix_len, group_size, key_bits, value_bits;
  int64_t key_payload_bh_stride;   /* bytes    */
  int64_t key_meta_bh_stride;      /* elements */
  int64_t key_residual_bh_stride;  /* elements */
  int64_t value_payload_bh_stride; /* bytes    */
  int64_t value_meta_bh_stride;    /* elements */
  int out_dtype;      /* 0: bf16 output (the query dtype), 1: fp32 output */
  int split_tokens;   /* > 0: tokens per split (rounded up to 32); 0: auto */
  int num_sms;        /* 0: query the current device */
  void* workspace; size_t workspace_bytes;   /* split partials */
  int* counters;      /* n_layers*batch*kv_heads ints, zero on entry */
  /* 1: the layers' query pointers are page-locked host memory the device
   * addresses directly (kvr_host_mapped).  Where the launch runs in
   * clusters (kvr_decode_cluster > 1) one CTA per (layer, b, kv head)
   * reads its queries across PCIe and shares them with the other splits
   * over distributed shared memory; otherwise every split reads them.
   * Zero-initialise the struct so the field is 0 when unused.              */
  int query_host_mapped;
} kvr_decode_args;

/* Key scales as fp16 pairs in the decode kernel's register order, for
 * kvr_layer_ptrs.key_scale_pairs.  No reference counterpart: a decode
 * lookup table derived from the stored bf16 scales
 * (packed_kv_cache.py:232-246), written once per key group when the
 * group is packed (pack_per_channel_grouped_affine, PackedLayer.commit).
 * Converts groups [group0, group0 + groups) of every (b,h) slab; `pairs`
 * has key_scale's layout ([bh][groups][D] 16-bit words, the given
 * bh stride).  head_dim in {64, 128}, key_bits in {2, 4, 8}.              */
typedef struct {
  const uint16_t* scale; int64_t scale_bh_stride;   /* bf16, elements */
  uint16_t* pairs; int64_t pairs_bh_stride;         /* fp16 pairs, elements */
  int bh, groups, group0, head_dim, key_bits;
} kvr_scale_pairs_args;
int kvr_key_scale_pairs(const kvr_scale_pairs_args* a, kvr_stream_t stream);

/* *flag = 1 if a decode on the current device has emitted a non-finite
 * output since the flag was last cleared (clear != 0 clears it), else 0.
 * Synchronises the device.  No reference counterpart: the reference
 * computes in fp32, where this kernel feeds the tensor cores fp16
 * operands.  Queries are scaled by an exact power of two to |q| < 64;
 * a key scale, a scaled query times a key scale, or a value scale at or
 * above 65504 is outside fp16's range, and such a decode's outputs are
 * non-finite.                                                             */
int kvr_decode_nonfinite(int* flag, int clear);

/* Fills the split count, workspace bytes and counter count for `a`
 * (workspace and counters ignored). */
int kvr_decode_plan(const kvr_decode_args* a, int* num_splits,
                    size_t* workspace_bytes, size_t* counter_count);
int kvr_decode_attention(const kvr_decode_args* a, kvr_stream_t stream);
/* The cluster size kvr_decode_attention would launch with on the current
 * device (1: no clusters; > 1: all splits of a (layer, b, kv head) form one
 * cluster).  No reference counterpart.                                     */
int kvr_decode_cluster(const kvr_decode_args* a, int* cluster);

/* Same as kvr_decode_attention for callers that cannot allocate device
 * memory (an FFI host without a CUDA allocator, a serving loop that must not
 * call cudaMalloc, a fixed memory budget).  No counterpart in the reference:
 * its decode path always allocates its split buffers with torch.
 * a->workspace and a->counters are ignored; the split scratch is a fixed
 * 4 MiB array compiled into the library, held by every GPU that loads it.
 * A problem whose plan needs more scratch than that returns
 * KVR_ERR_WORKSPACE.  The first call on a device looks up the array's
 * address (make it before any stream capture on that device); host threads
 * may make that first call at the same time.  Every call shares the array
 * and clears its counters; calls that overlap on the GPU race.             */
int kvr_decode_attention_noalloc(const kvr_decode_args* a, kvr_stream_t stream);

/* kvr_decode_attention with the sequence and prefix lengths read from
 * device memory at run time (lengths as for kvr_append_lengths).  a
 * describes the capacity: a->seq_len = value rows the buffers hold (the
 * split plan covers them; splits past the live length add nothing),
 * a->prefix_len = key rows the payload/metadata buffers hold (a multiple
 * of group_size), residual_capacity = rows of the BF16 key residual
 * buffer.  The live lengths are clamped to those capacities.  No reference
 * counterpart.                                                             */
int kvr_decode_attention_lengths(const kvr_decode_args* a, const int* lengths, int residual_capacity,
                                 kvr_stream_t stream);

/* The same decode on the CUDA cores (fp32 FMA, no tensor cores): the
 * measured A/B baseline the tensor-core kernel is adopted against.  Same
 * arguments; a->workspace must hold kvr_decode_simt_workspace(a) bytes
 * (split partials; counters unused; 0 = invalid or unsupported).
 * Supported: (D, key bits, value bits, HQ/HKV) in {(128,4,4,6), (128,2,2,6),
 * (128,4,4,4), (64,8,4,4), (64,4,8,4)}, group_size a power of two >= 32.
 * No reference counterpart (the reference's Triton kernels are the
 * CUDA-core formulation).                                                  */
size_t kvr_decode_simt_workspace(const kvr_decode_args* a);
int kvr_decode_attention_simt(const kvr_decode_args* a, kvr_stream_t stream);

/* One decode step with the append fused in: the new token's key row
 * (k_new, [B, HKV, 1, D] bf16) goes to the BF16 residual and its value row
 * (v_new) is quantized per token, exactly as kvr_append_lengths with n = 1,
 * by the decode launch itself -- the CTA whose split holds the new token
 * stores it before reading its first chunk -- and the decode then attends
 * over the sequence including it; lengths advance by one (their last CTA to
 * read them moves them).  a and residual_capacity as for
 * kvr_decode_attention_lengths, with n_layers == 1; a step past a capacity
 * sets lengths[2] and decodes without appending.  Replaces the two launches
 * of kvr_append_lengths + kvr_decode_attention_lengths (PackedLayer.append
 * then the attention call, packed_review.py:23-31 and :78).              */
int kvr_decode_step(const kvr_decode_args* a, const uint16_t* k_new, const uint16_t* v_new, int* lengths,
                    int residual_capacity, kvr_stream_t stream);

/* LSE merge of externally produced partials (the cross-GPU token split):
 * parts: n_parts blocks of [rows] (m, l) pairs and [rows, D] unnormalised
 * outputs, m in log2 units; out[rows, D] bf16 = sum_p 2^(m_p-M) o_p /
 * sum_p 2^(m_p-M) l_p.  Rows with no mass are written as zero.            */
int kvr_lse_merge(const float* part_ml, const float* part_o, int n_parts,
                  int rows, int head_dim, uint16_t* out, kvr_stream_t stream);

/* Partial decode for one shard of the token axis: same as
 * kvr_decode_attention but over tokens [token_begin, token_end) only, with
 * one split per (layer, b, kv head); writes (m, l) pairs to part_ml
 * [n_layers*B*HQ] and unnormalised outputs to part_o [n_layers*B*HQ, D]
 * instead of the final output (for kvr_lse_merge after an all-gather).     */
int kvr_decode_partial(const kvr_decode_args* a, int token_begin, int token_end,
                       float* part_ml, float* part_o, kvr_stream_t stream);

/* ----------------------------------------- cross-GPU exchange + merge
 * Sequence-split decode across GPUs (no reference counterpart: the
 * reference runs on one GPU): every rank holds partials (m, l, o) of its
 * token shard from kvr_decode_partial; kvr_exchange_merge stores them into
 * every peer's receive buffer over NVLink (CUDA IPC peer mappings), signals
 * the peers, waits for theirs (bounded by timeout_ns; a time-out sets
 * *error) and writes the LSE merge of all ranks as bf16 out[rows, D].
 * Receive buffer of each rank: floats [2][world][rows*(2+D)] (halves
 * alternate by step; per source: (m, l) [rows][2] then o [rows][D]) then
 * int signal[world] at byte offset 8*world*rows*(2+D), 256 bytes reserved.
 * epoch, counter and error start at zero; every rank makes the same calls
 * in the same order.  The caller's partials for step n (n = 1, 2, ...) go
 * into its own buffer's half n % 2, source slot rank.                      */
typedef struct {
  int world, rank, rows, head_dim;
  float* const* recv;   /* device array [world]: each rank's receive buffer, as mapped here */
  int* const* signal;   /* device array [world]: each rank's signal words, as mapped here */
  int* epoch;           /* this rank, device: exchanges completed */
  int* counter;         /* this rank, device: arrival counter */
  int* error;           /* this rank, device: non-zero after a wait timed out */
  uint16_t* out;        /* bf16 [rows, head_dim] */
  long long timeout_ns;
  int mode;             /* kvr_decode_partial_exchange: 0 rows to every rank, 1 rows to their owner */
} kvr_exchange_args;
int kvr_exchange_merge(const kvr_exchange_args* a, kvr_stream_t stream);

/* Delivered mode (head_dim 64 or 128, world <= 8): kvr_decode_partial_exchange
 * runs the decode over [token_begin, token_end) and, instead of writing
 * partials locally, stores each finished row straight into this rank's
 * slot of every rank's receive area as 8-byte words (value bits, epoch),
 * each written whole (the low-latency protocol NCCL publishes as "LL"):
 * uint32 words [2 halves][world sources][rows][2 + D][2] at byte offset
 * 256 of each signal area, row = (m, l, o[0..D)), half = step % 2.  No
 * fence and no flag: kvr_exchange_merge_delivered reads every source's
 * words for a row until all carry this step's epoch (bounded by
 * timeout_ns; a time-out sets *error), merges the row from local memory
 * and advances the epoch.  The buffer of each rank is then
 * 8*world*rows*(2+D) + 256 + 16*world*rows*(2+D) bytes.  x->rows must be
 * n_layers*batch*q_heads; recv, out, counter and timeout_ns are not used
 * by the decode.                                                           */
int kvr_decode_partial_exchange(const kvr_decode_args* a, int token_begin, int token_end,
                                const kvr_exchange_args* x, kvr_stream_t stream);
int kvr_exchange_merge_delivered(const kvr_exchange_args* a, kvr_stream_t stream);

/* Owner mode (x->mode = 1; head_dim 64 or 128, world <= 8): a reduce-scatter
 * of the partials, then an all-gather of the merged rows, both as tagged
 * words.  kvr_decode_partial_exchange stores each row only into the
 * receive area of its owner, rank row % world (same layout as above).
 * kvr_exchange_merge_owned waits for every source's words of the rows this
 * rank owns (bounded), merges them into out and stores each merged row as
 * words (bf16 pair, epoch) into every peer's final area: uint32 words
 * [2 halves][rows][D] after the receive area.  kvr_exchange_gather_owned
 * then waits for the other ranks' rows there (bounded), copies them into
 * out and advances the epoch.  Each rank sends about 1/world of the
 * delivered mode's bytes, for one more hop.  The buffer of each rank is
 * 8*world*rows*(2+D) + 256 + 16*world*rows*(2+D) + 8*rows*D bytes.         */
int kvr_exchange_merge_owned(const kvr_exchange_args* a, kvr_stream_t stream);
int kvr_exchange_gather_owned(const kvr_exchange_args* a, kvr_stream_t stream);

/* Receive buffers shared between processes: device memory from cudaMalloc
 * (zeroed) with a 64-byte CUDA IPC handle; a peer maps it with
 * kvr_exchange_open and unmaps it with kvr_exchange_close.                 */
int kvr_exchange_alloc(size_t bytes, void** ptr, unsigned char* handle);
int kvr_exchange_open(const unsigned char* handle, void** ptr);
int kvr_exchange_close(void* ptr);
int kvr_exchange_free(void* ptr);

#ifdef __cplusplus
}
#endif
#endif /* KVR_H_ */
