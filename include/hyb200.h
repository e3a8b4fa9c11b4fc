/*
 * hyb200.h — C ABI of the B200 (sm_100a) chunk-causal cached attention path.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * launches on the caller's CUDA stream and returns an int status
 * (HYB_OK == 0, negative on error; hyb_last_error() gives the message).
 * Nothing here allocates device memory: per-call scratch comes from a
 * caller-provided workspace whose size hyb_cached_attention_workspace_bytes()
 * reports.  No torch types cross this boundary.
 *
 * Reference interfaces replaced (paths relative to the Hy-Nomas project):
 *   hyb_kv_append_pair        <- quantize_kv_pair_into / quantize_kv_into / _quantize_rows
 *                                hymm/models/dit/modules/int8_kv_cache.py:125-179, :22-58
 *                                (HYB_FMT_INT8 exact; HYB_FMT_E4M3 is the same rule with a
 *                                448 denominator and an e4m3 RNE cast)
 *   hyb_kv_dequant            <- dequantize_kv / _dequantize_rows
 *                                hymm/models/dit/modules/int8_kv_cache.py:182-205, :61-89
 *   hyb_cached_attention      <- causal_attention_with_cache_mp, single rank part (history
 *                                decode, K/V composition, masks, kernel, pad)
 *                                hymm/models/dit/nomas_cpt.py:335-884 (steps 2-6 of the call),
 *                                and the sm_100 incumbent CacheStaging.__call__ +
 *                                compact_kv reactor/hy_nomas_cache.py:192-338, :48-73
 *   hyb_attn_fwd              <- the kernel call inside it: flash_attn_varlen_func (FA3/FA4)
 *                                nomas_cpt.py:786-829, magi flex_flash_attn_func with the
 *                                chunk-causal ranges of attention/magi_attn.py:290-309
 *   hyb_lse_merge             <- flash_attn_fwd_out_correction / _softmax_lse_correction
 *                                hymm/models/dit/modules/attention/dynamic_ring_attention.py:86-105
 *   hyb_part_scatter +        <- the same merge for sequence-parallel attention over a
 *   hyb_merge_partials           sequence-sharded (KV-stationary) cache: partial rows written to
 *                                their owner ranks by the attention epilogue, merged there
 *   hyb_ulysses_pack_qkv      <- pack_qkv + all_to_all_qkv send-side layout
 *                                reactor/hy_nomas_fusions.py:56-78, hymm/distributed/communications.py:270-280
 *   hyb_ulysses_unpack_o      <- _all_to_all_4D(scatter_idx=1, gather_idx=2) receive-side layout
 *                                hymm/distributed/communications.py:158-200
 */
#ifndef HYB200_H_
#define HYB200_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HYB_ABI_VERSION 5

/* status codes */
#define HYB_OK 0
#define HYB_ERR_INVALID_ARG (-1)   /* bad shape / stride / pointer / size (ValueError) */
#define HYB_ERR_UNSUPPORTED (-2)   /* head_dim != 128, dtype, arch (RuntimeError) */
#define HYB_ERR_CUDA (-3)          /* CUDA runtime error (RuntimeError) */
#define HYB_ERR_TIMEOUT (-4)       /* a bounded device-side wait expired (RuntimeError) */
#define HYB_ERR_NONFINITE (-5)     /* non-finite K/V handed to the quantiser (ValueError) */
#define HYB_ERR_CAPACITY (-6)      /* write past cache capacity (ValueError) */
#define HYB_ERR_WORKSPACE (-7)     /* workspace too small (RuntimeError) */

/* element formats */
#define HYB_FMT_BF16 0   /* plain bf16 values */
#define HYB_FMT_E4M3 1   /* float8_e4m3fn codes + fp32 per-(token, head) scale */
#define HYB_FMT_INT8 2   /* int8 codes + fp32 per-(token, head) scale (reference format) */

/* device status bits written by kernels into a caller-provided int32 */
#define HYB_DEV_TIMEOUT 0x1
#define HYB_DEV_NONFINITE 0x2

/* A [B, L, H, D] tensor view with unit stride on D (strides in elements).
 * For HYB_FMT_E4M3 / HYB_FMT_INT8, `scale` is the fp32 [B, L, H(, 1)] scale tensor. */
typedef struct hyb_tensor4 {
  const void* data;
  int32_t fmt;
  int32_t pad_;
  int64_t s_b, s_t, s_h;
  const float* scale;
  int64_t ss_b, ss_t, ss_h;
} hyb_tensor4;

/* One cached-attention call on one rank (after any Ulysses exchange).
 * Keys attended by every query: [visible history | current image | current text].
 * Image query i sees image key j iff j / group_tokens <= i / group_tokens
 * (group_tokens == 0: the whole chunk is bidirectional, the reference's cached path).
 * Text queries see every visible key.  History key t is visible iff cache_mask[b, t];
 * text key t iff text_mask[b, t].  Output rows of masked text queries are zero
 * (the flash3 path's pad_tokens semantics, nomas_cpt.py:823-829). */
/* Partial rows scattered to their owners: sequence-parallel attention over a sequence-sharded
 * ("KV-stationary") cache.  Every rank attends all queries of the chunk to the keys it holds;
 * the epilogue writes each query row's partial result for its key slice (O / l in fp32 and the
 * natural-log LSE, -inf when the slice saw no visible key) straight into the buffers of the rank
 * that owns the row (peer-mapped memory), where hyb_merge_partials combines the partials.
 * Image query q belongs to rank q / rows at local row q % rows; text query t is written to every
 * rank, at local row rows + t.  Owner buffers (device arrays of `ranks` pointers, each the
 * owner's buffer as mapped on the calling rank): o fp32 [count, B, H, rows + txt, D], lse fp32
 * [count, B, H, rows + txt].  This launch writes partial indices [index0, index0 + slices): every
 * query pair's key tiles are cut into exactly `slices` slices (1..16).  No reference counterpart
 * in code (the reference passes K/V around a ring, dynamic_ring_attention.py:115-286; its merge
 * formula, :86-105, is the one applied here). */
typedef struct hyb_part_scatter {
  float* const* o;
  float* const* lse;
  int32_t ranks, rows, index0, count, slices, pad_;
} hyb_part_scatter;

typedef struct hyb_cached_attn_args {
  int32_t abi_version;     /* HYB_ABI_VERSION */
  int32_t B, H, D;         /* batch, heads on this rank, head_dim (128) */
  int32_t cache_batch;     /* batch of the history tensors: B, or 1 (read-only broadcast) */
  int32_t valid_len;       /* history tokens [0, valid_len) read from hist_k/hist_v; at most their
                              capacity (views carry no extent, so this is the caller's to ensure) */
  int32_t img_len, txt_len;
  int32_t attend_txt;      /* 1: current text keys are attended (cache_txt or update_cache) */
  int32_t group_tokens;    /* block-causal granularity in tokens (G frames x tokens/frame), 0 = off */
  float softmax_scale;     /* <= 0 selects 1/sqrt(D) */
  int32_t q_pos0, k_pos0;  /* global positions of image query 0 / image key 0 for the block-causal
                              rule: query i sees key j iff (k_pos0+j)/G <= (q_pos0+i)/G (0, 0 for a
                              chunk attending to itself; ring steps pass shard offsets) */
  hyb_tensor4 hist_k, hist_v;                 /* cache: BF16 / E4M3 / INT8 */
  hyb_tensor4 img_q, img_k, img_v;            /* Q BF16 [B, img_len, H, D]; K/V BF16, E4M3 or INT8 */
  hyb_tensor4 txt_q, txt_k, txt_v;            /* BF16 [B, txt_len, H, D] */
  const int32_t* hist_rows; /* [valid_len] cache row of composed history position t, or NULL
                               (identity); sink + sliding-window rings use it.  Every row must lie
                               in [0, capacity of hist_k); the device does not check it */
  const uint8_t* cache_mask; int64_t cache_mask_sb;  /* bool [cache_batch, cap] (cache rows) or NULL */
  const uint8_t* text_mask;  int64_t text_mask_sb;   /* bool [B, txt_len] or NULL */
  void* out_img; int64_t oi_sb, oi_st, oi_sh;        /* bf16 [B, img_len, H, D] */
  int64_t oi_seg, oi_sseg; /* image row t at (t / oi_seg) * oi_sseg + (t % oi_seg) * oi_st;
                              oi_seg <= 0 means img_len (no segmentation) */
  void* out_txt; int64_t ot_sb, ot_st, ot_sh;        /* bf16 [B, txt_len, H, D] */
  float* lse;              /* fp32 [B, H, img_len + txt_len] natural-log LSE, or NULL */
  void* workspace; int64_t workspace_bytes;
  int32_t* dev_status;     /* int32 on the device, OR-ed with HYB_DEV_* bits, or NULL */
  int32_t img_k_len;       /* current image keys [B, img_k_len, H, D] in img_k/img_v; 0 means
                              img_len (the chunk attends to itself).  A rank of a KV-stationary
                              schedule passes all queries of the chunk and its own keys */
  const hyb_part_scatter* scatter;  /* NULL, or: partial rows go to their owners (out_img/out_txt
                                       unused, no merge here) */
  /* Pre-decoded history (ABI 5), or NULL: the call decodes hist_k / hist_v through hist_rows.
     When staged_k is set, history key t (t < valid_len) is row t of staged_k / staged_v, bf16 K
     and fp16 V [B, H, staged_pitch, D] holding the values the call's own decode would produce
     (a cache that decodes each appended frame once, see hyb_decode_rows); hist_k, hist_v and
     hist_rows are not read, cache_mask is indexed by t, and the current image and text keys
     are staged into rows [valid_len, valid_len + img_k_len + txt_len) of the same buffers, so
     staged_pitch must cover them.  The order of the history rows is free: attention is a sum
     over the set of visible keys. */
  void* staged_k;
  void* staged_v;
  int64_t staged_pitch;
} hyb_cached_attn_args;

/* Decode n rows of a quantised K/V pair (E4M3 / INT8 views [B, n, H, D] with their scales)
 * into head-major rows [row0, row0 + n) of dst_k (bf16) and dst_v (fp16 holding the same bf16
 * value) [B, H, pitch, D]: value for value the decode hyb_cached_attention applies to history
 * rows (bf16(code * scale), dequantize_kv of int8_kv_cache.py:182-205).  A cache that decodes
 * each frame once when it is appended passes these buffers as staged_k / staged_v.  No
 * reference counterpart: the reference decodes the whole cache on every call
 * (nomas_cpt.py:529-531). */
int hyb_decode_rows(int32_t B, int32_t n, int32_t H, int32_t D, const hyb_tensor4* src_k,
                    const hyb_tensor4* src_v, void* dst_k, void* dst_v, int64_t pitch, int64_t row0,
                    void* stream);

/* Workspace bytes of hyb_cached_attention; staged != 0 for a call with staged_k set (no
 * K/V staging area: the caller's buffers hold it). */
int64_t hyb_cached_attention_workspace_bytes_ex(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                                int32_t img_len, int32_t txt_len, int32_t attend_txt,
                                                int32_t staged);

/* Library identity. */
int hyb_version(void);
/* Copies the calling thread's last error message (NUL-terminated). Returns its length. */
int hyb_last_error(char* buf, size_t len);
/* 1 if the current device is sm_100 (B200/GB200) and the kernels can run, else 0. */
int hyb_device_supported(void);

/* Quantise-on-write of a K/V pair into a per-token-per-head scaled cache.
 * Sources: bf16 [B, L, H, D] rows t < L from src_k/src_v, then (when L2 > 0) rows
 * L <= t < L + L2 from src_k2/src_v2 (image tokens followed by text tokens, without
 * concatenating them first).  Codes go to token offset `start` of [B, cap, H, D];
 * scales fp32 [B, cap, H, 1].  Scale = absmax/127 (INT8) or absmax/448 (E4M3), 1 for an
 * all-zero row; codes use IEEE division.  dev_status (may be NULL) gets
 * HYB_DEV_NONFINITE if any input was not finite. */
int hyb_kv_append_pair(int32_t fmt, int32_t B, int32_t L, int32_t H, int32_t D, int64_t cap,
                       int64_t start,
                       const hyb_tensor4* src_k, const hyb_tensor4* src_v,
                       int32_t L2, const hyb_tensor4* src_k2, const hyb_tensor4* src_v2,
                       void* dst_k, void* dst_v, int64_t d_sb, int64_t d_st, int64_t d_sh,
                       float* scale_k, float* scale_v, int64_t s_sb, int64_t s_st, int64_t s_sh,
                       int32_t* dev_status, void* stream);

/* Finite check of a bf16 [B, L, H, D] tensor; ORs HYB_DEV_NONFINITE into dev_status. */
int hyb_check_finite(const hyb_tensor4* src, int32_t B, int32_t L, int32_t H, int32_t D,
                     int32_t* dev_status, void* stream);

/* Decode the valid prefix of a quantised cache into bf16 [B, valid, H, D] (contiguous). */
int hyb_kv_dequant(const hyb_tensor4* src, int32_t B, int32_t valid, int32_t H, int32_t D,
                   void* dst, void* stream);

/* Workspace bytes needed by hyb_cached_attention for these sizes. */
int64_t hyb_cached_attention_workspace_bytes(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                             int32_t img_len, int32_t txt_len, int32_t attend_txt);

/* Byte offsets of the staging workspace of hyb_cached_attention for these sizes on the
 * current device (the key-slice count kv_splits depends on its multiprocessor count). */
typedef struct hyb_workspace_layout {
  int64_t q, k, v, kbits, qbits, part_o, part_lse, total;
  int32_t Lq, Lk, kwords, qwords, kv_splits, pad_;
} hyb_workspace_layout;
int hyb_cached_attention_workspace_layout(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                          int32_t img_len, int32_t txt_len, int32_t attend_txt,
                                          hyb_workspace_layout* out);

/* The whole single-rank cached attention (stage + tcgen05 attention kernel). */
int hyb_cached_attention(const hyb_cached_attn_args* args, void* stream);

/* Attention kernel alone over staged head-major bf16 tensors:
 * q [B, H, Lq, D], k/v [B, H, Lk, D] (contiguous).  Key j < hist_len is history,
 * [hist_len, hist_len + img_len) current image (block-causal), the rest text.
 * kbits: [B, kwords] visibility bitmap of keys; qbits: [B, qwords] query validity. */
typedef struct hyb_attn_args {
  int32_t abi_version;
  int32_t B, H, D, Lq, Lk, hist_len, img_len, group_tokens;
  float softmax_scale;
  int32_t q_pos0, k_pos0;   /* as in hyb_cached_attn_args */
  int32_t img_k_len;        /* image keys [hist_len, hist_len + img_k_len); 0 means img_len */
  int32_t q_seg, q_pos1;    /* two-segment query positions (zig-zag ring shards): image query i
                               is at q_pos0 + i for i < q_seg, else at q_pos1 + (i - q_seg);
                               q_seg <= 0 means one segment */
  int32_t k_seg, k_pos1;    /* the same for image keys; positions must increase
                               (k_pos1 >= k_pos0 + k_seg) so that every query sees a key prefix */
  int32_t pad1_;
  const void* q; const void* k; const void* v;
  const uint32_t* kbits; int32_t kwords;
  const uint32_t* qbits; int32_t qwords;
  void* out_img; int64_t oi_sb, oi_st, oi_sh;
  int64_t oi_seg, oi_sseg;   /* image row t lands at (t / oi_seg) * oi_sseg + (t % oi_seg) * oi_st */
  void* out_txt; int64_t ot_sb, ot_st, ot_sh;
  float* lse;
  int32_t* dev_status;
  int32_t kv_splits;         /* >1: each query pair's key tiles are split into this many slices */
  int32_t v_f16;             /* 1: v holds fp16 values and the softmax weights P are rounded to fp16
                                (11-bit significand) for P.V; 0: v and P in bf16 (8-bit significand).
                                bf16 values convert to fp16 exactly within fp16's range */
  float* part_o;             /* fp32 [kv_splits, B, H, Lq, D] partial rows (kv_splits > 1) */
  float* part_lse;           /* fp32 [kv_splits, B, H, Lq] partial LSE (kv_splits > 1) */
  /* Running output of a ring (KV-passing) schedule, or NULL.  With acc_o set, every query is an
     image query (Lq == img_len) and this launch's rows are merged by log-sum-exp with
     acc_o fp32 [B, Lq, H, D] / acc_lse fp32 [B, H, Lq] (natural log).  acc_mode bit 0: merge
     with the accumulator's contents (else this launch starts it); bit 1: final step — write
     the merged rows as bf16 to out_img (and the LSE to lse when non-NULL) instead of acc_o. */
  float* acc_o;
  float* acc_lse;
  int32_t acc_mode;
  int32_t pad2_;
  const hyb_part_scatter* scatter;  /* NULL, or: partial rows go to their owners (see above);
                                       kv_splits and part_o/part_lse are then unused */
} hyb_attn_args;
int hyb_attn_fwd(const hyb_attn_args* args, void* stream);

/* Launch plan of hyb_attn_fwd for these arguments on a device with `sms` multiprocessors
 * (sms <= 0: the current device): splits[i] = number of key slices query pair i (rows
 * [256 i, 256 i + 256)) is cut into, for i < n; at most args->kv_splits.  Returns the number of
 * query pairs, or a negative status.  Host only, no device work.  No reference counterpart
 * (launch planning of this kernel: a heavy pair is cut into more slices so that every CTA of
 * the launch gets about the same number of key tiles). */
int hyb_attn_work_plan(const hyb_attn_args* args, int32_t sms, int32_t* splits, int32_t n);

/* Decode a K/V block (or one Q tensor) [B, L, H, D] in BF16, E4M3 or INT8 with per-(token,
 * head) scales into head-major bf16 [B, H, L, 128], the operand layout hyb_attn_fwd reads
 * (codes times scale in fp32, one rounding, as dequantize_kv).  src_v and dst_v may both be
 * NULL (one tensor).  Replaces, for callers that keep operands staged across calls (the ring),
 * dequantize_kv + torch.cat of the reference's cached path (int8_kv_cache.py:182-205,
 * nomas_cpt.py:614-649) and the q/k/v layout copies before flash_attn_func in
 * dynamic_ring_attention.py:45-83. */
int hyb_stage_head_major(int32_t B, int32_t L, int32_t H, int32_t D, const hyb_tensor4* src_k,
                         const hyb_tensor4* src_v, void* dst_k, void* dst_v, void* stream);

/* Sequence-parallel K/V blocks of P ranks -> head-major bf16 K and V [H, L, 128] of the whole
 * sequence.  Block r (blocks[r], as mapped here) is [K codes | V codes | K scales | V scales]
 * for Lmax rows of H heads; position pos in chunk c ([bounds[c], bounds[c+1])) is row
 * row0[c] + pos - bounds[c] of block owner[c].  Decode as hyb_kv_dequant; with v_f16 = 1 the
 * decoded bf16 V is stored as fp16 (exact), the operand of hyb_attn_fwd with v_f16 = 1.
 * Replaces the per-step kv buffers of the reference ring (dynamic_ring_attention.py:115-286). */
int hyb_ring_gather_stage(int32_t P, int32_t fmt, int32_t L, int32_t H, int32_t D, int32_t Lmax,
                          const void* const* blocks, int32_t nchunks, const int32_t* bounds,
                          const int32_t* owner, const int32_t* row0, void* out_k, void* out_v,
                          int32_t v_f16, void* stream);

/* Key-visibility bitmap for hyb_attn_fwd with keys [0, Lk) of every batch row visible:
 * bits [B, kwords] uint32.  No reference counterpart (the reference ring attends every key of
 * a block; flash_attn_func takes no key mask). */
int hyb_fill_key_bits(int32_t B, int32_t Lk, int32_t kwords, uint32_t* bits, void* stream);

/* Ring merge of two partial attentions (fp32 LSE in natural log):
 * lse = log(exp(lse_a) + exp(lse_b)); out = out_a * exp(lse_a - lse) + out_b * exp(lse_b - lse).
 * out_acc/lse_acc [rows, H, D]/[H, rows] are updated in place with (out_b, lse_b). */
int hyb_lse_merge(int32_t rows, int32_t H, int32_t D,
                  float* out_acc, float* lse_acc, const void* out_b, int32_t out_b_fmt,
                  const float* lse_b, void* stream);

/* Owner side of hyb_part_scatter: the `count` partials of each row of this rank's buffers
 * (o [count, B, H, rows + txt_rows, D], lse [count, B, H, rows + txt_rows]) merged by
 * log-sum-exp (dynamic_ring_attention.py:86-105) into bf16 out_img [B, rows, H, D] and out_txt
 * [B, txt_rows, H, D] (element strides).  A text row whose text_mask entry (bool [B, txt_rows],
 * or NULL: all valid) is false, and a row that no partial saw, is written as zeros (the
 * reference's padded text queries, nomas_cpt.py:807-829).  lse (fp32 [B, H, rows + txt_rows]) may
 * be NULL. */
int hyb_merge_partials(int32_t count, int32_t B, int32_t H, int32_t D, int32_t rows, int32_t txt_rows,
                       const float* part_o, const float* part_lse,
                       void* out_img, int64_t oi_sb, int64_t oi_st, int64_t oi_sh,
                       void* out_txt, int64_t ot_sb, int64_t ot_st, int64_t ot_sh,
                       const uint8_t* text_mask, int64_t text_mask_sb, float* lse, void* stream);

/* ---------------------------------------------------------------------------------------
 * Peer-memory exchange for Ulysses sequence parallelism (one process per GPU).  Buffers are
 * device allocations shared with CUDA IPC; every rank maps every other rank's buffers.  The
 * push calls write this rank's slices straight into the destination ranks' buffers over
 * NVLink and end with a device-side flag barrier (bounded: a rank that never arrives makes
 * the others report HYB_DEV_TIMEOUT in dev_status after ~2 s instead of hanging).  They
 * replace the all_to_all_single / all_gather collectives of all_to_all_qkv, all_to_all_4D
 * and all_gather (hymm/distributed/communications.py:66-200, :270-280, :410-421) with one
 * kernel each; the bytes land in the same layouts.
 * ------------------------------------------------------------------------------------- */
typedef struct hyb_peer_sync {
  int32_t* flags[64];      /* every rank's flag array int32[P] (peer-shared), as mapped here */
  uint32_t* state;         /* this rank's uint32[2] (blocks arrived, epoch), zero-initialised */
  int32_t* dev_status;     /* int32 status word, OR-ed with HYB_DEV_TIMEOUT, or NULL */
} hyb_peer_sync;

/* cudaMalloc(bytes) zero-filled, and its IPC handle (64 bytes) for the other ranks. */
int hyb_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
/* Map another rank's buffer (IPC handle from hyb_peer_alloc) into this process. */
int hyb_peer_open(const void* ipc_handle, void** peer_ptr);
int hyb_peer_close(void* peer_ptr);
int hyb_peer_free(void* ptr);

/* q, k, v bf16 [B, Ls, H, D] -> rank d's receive buffer recv[d] [P(src), Ls, 3B, H/P, D] at
 * slot src = rank (heads [d*H/P, (d+1)*H/P)), then the barrier.  Same bytes as the receive
 * side of all_to_all_qkv (communications.py:270-280) with equal sequence lengths. */
int hyb_ulysses_push_qkv(int32_t P, int32_t rank, int32_t B, int32_t Ls, int32_t H, int32_t D,
                         const hyb_tensor4* q, const hyb_tensor4* k, const hyb_tensor4* v,
                         void* const* recv, const hyb_peer_sync* sync, void* stream);

/* This rank's attention output for its H/P heads -> every rank's final layout: o_send
 * [P(dst), H/P, Ls, B, D] (the layout the attention epilogue writes) to out[d] [B, Ls, H, D]
 * at heads [rank*H/P, ...); text rows txt [B, Lt, H/P, D] to every txt_out[d] [B, Lt, H, D];
 * then the barrier.  Replaces all_to_all_4D(scatter 1, gather 2) of the image rows and the
 * head all_gather of the text rows (communications.py:260-267, :410-421; nomas_cpt.py:864-872). */
int hyb_ulysses_push_o(int32_t P, int32_t rank, int32_t B, int32_t Ls, int32_t Lt, int32_t H, int32_t D,
                       const void* o_send, const hyb_tensor4* txt, void* const* out, void* const* txt_out,
                       const hyb_peer_sync* sync, void* stream);

/* The device barrier alone (one block): each rank arrives once its stream reaches the launch
 * and waits, bounded, for every other rank (HYB_DEV_TIMEOUT in dev_status after ~2 s).  No
 * reference counterpart (the reference's NCCL send/recv pairs each transfer with its own
 * receive, dynamic_ring_attention.py:45-83); ring_attention's all-gather schedule launches it
 * before pushing a call's blocks, so no rank overwrites a block a peer is still decoding. */
int hyb_peer_barrier(int32_t P, int32_t rank, const hyb_peer_sync* sync, void* stream);

/* All-gather contribution over peer memory: `bytes` (a multiple of 16) from src to dst[d] on
 * every rank d (skipping dst[d] == src), then the barrier.  The ring schedule of
 * ring_attention passes its e4m3 K/V blocks this way (every block to every rank at once over
 * NVSwitch instead of one neighbour hop per step: flash_attn_p2p_communicate,
 * dynamic_ring_attention.py:45-83). */
int hyb_peer_push_bytes(int32_t P, int32_t rank, const void* src, int64_t bytes, void* const* dst,
                        const hyb_peer_sync* sync, void* stream);
/* The same on at most max_blocks blocks of 256 threads (<= 0: as many as the bytes need), so
 * that a kernel on another stream (the own-block attention of the overlapped ring schedule)
 * runs on the other SMs while the push crosses NVLink. */
int hyb_peer_push_bytes_n(int32_t P, int32_t rank, const void* src, int64_t bytes, void* const* dst,
                          const hyb_peer_sync* sync, int32_t max_blocks, void* stream);

/* Ulysses send-side pack (sequence -> heads): q, k, v bf16 [B, Ls, H, D] -> send buffer
 * [P, Ls_max, nsrc*B, H/P, D] (the all_to_all_qkv layout, padding rows zeroed).
 * k == v == NULL packs q alone (nsrc = 1, the all_to_all_4D(scatter 2, gather 1) layout). */
int hyb_ulysses_pack_qkv(int32_t P, int32_t B, int32_t Ls, int32_t Ls_max, int32_t H, int32_t D,
                         const hyb_tensor4* q, const hyb_tensor4* k, const hyb_tensor4* v,
                         void* send, void* stream);

/* Ulysses send-side pack of O (heads -> sequence): x bf16 [B, L, H/P, D] with
 * L = sum(lens[0..P)) -> send buffer [P, H/P, Ls_max, B, D], padding rows zeroed. */
int hyb_ulysses_pack_o(int32_t P, int32_t B, const int32_t* lens, int32_t Ls_max, int32_t Hp, int32_t D,
                       const hyb_tensor4* x, void* send, void* stream);

/* Ulysses receive-side unpack of O: recv [P, H/P, Ls_max, B, D] -> out [B, Ls, H, D] strided. */
int hyb_ulysses_unpack_o(int32_t P, int32_t B, int32_t Ls, int32_t Ls_max, int32_t H, int32_t D,
                         const void* recv, void* out, int64_t o_sb, int64_t o_st, int64_t o_sh,
                         void* stream);

/* hyb_cached_attention for callers that cannot allocate device memory (no counterpart in
 * the reference).  Same arguments and results; args->workspace / workspace_bytes are
 * ignored and the staging scratch is a fixed 64 MiB array of static device memory inside
 * this library, which every GPU that loads the library holds until the process exits.
 * Sizes whose scratch (hyb_cached_attention_workspace_bytes) exceeds 64 MiB are rejected
 * with HYB_ERR_WORKSPACE; negative sizes with HYB_ERR_INVALID_ARG.  The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress) with that device current,
 * and so does the first call in a context created anew after a device reset; make those first
 * calls before any stream capture.  The function calls no allocator.  All calls on a device share the one
 * array, so calls that can overlap on the GPU (different streams, or concurrent host
 * threads) race on it and must be serialised by the caller. */
int hyb_cached_attention_noalloc(const hyb_cached_attn_args* args, void* stream);

/* Diagnostic: y[i] = the FMA-pipe exp2 approximation the attention softmax uses for a
 * share of its exponentials (no reference counterpart; used by the accuracy test). */
int hyb_exp2_poly_eval(const float* x, float* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HYB200_H_ */
