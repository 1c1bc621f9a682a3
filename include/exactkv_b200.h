/*
 * exactkv_b200 — C ABI of the B200 (sm_100a) kernels for the exactkv hot path.
 *
 * The library (exactkv_b200/libexactkv_b200.so) replaces the Triton module
 * exactkv/kernels.py of the reference. Every entry point takes plain device
 * pointers, element counts and strides, the CUDA device index and a
 * cudaStream_t passed as `void *`. Nothing here allocates device memory: the
 * caller owns every buffer, including the split-K workspace. Work is enqueued
 * on `stream` and nothing synchronises.
 *
 * Outputs (`out` of the attention and merge entries) may also be pinned host
 * memory mapped into the device's address space at the same address (any
 * cudaHostAlloc / cudaHostRegister allocation under unified addressing): the
 * merge kernel then writes the result straight to the host over PCIe, with no
 * separate device-to-host copy. Other host memory is rejected (EXK_EARG).
 *
 * Return value: 0 on success, a positive cudaError_t from the launch, or a
 * negative EXK_E* argument error (exk_error_string() describes every code).
 * Faults found by the kernels themselves (a spin-wait that ran out of time, a
 * raw-pool index past the pool) are written as a nonzero EXK_S* code to the
 * caller's device status word, which the caller reads when it next syncs.
 *
 * Compressed format (per 16-token page, per KV head, per channel; D = 128):
 *   sm      uint8 [B, TS, H, 128]     sign bit | 7 mantissa bits, unchanged
 *   code    uint8 [B, TS, H, 64]      4-bit exponent offsets; byte j holds
 *                                     channel j (low nibble) and j+64 (high)
 *   base    uint8 [B, TS/16, H, 128]  bit 7: the group holds zeros (code 0 =
 *                                     exponent 0); bits 0-6: exponent base
 *   rowmask int32 [B, TS/16, H]       bit p: token p of the page is raw
 *   rowoff  int32 [B, TS/16, H]       pool index of the page's first raw row
 *   raw     bf16  [rows, 128]         raw rows; a page's raw rows are adjacent
 * (reference: exactkv/codec.py:10-19, allocation exactkv/cache.py:24-32).
 */
#ifndef EXACTKV_B200_H
#define EXACTKV_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXK_HEAD_DIM 128
#define EXK_PAGE 16

/* argument errors (negative return values) */
#define EXK_EARG      (-1)  /* shape or count out of range */
#define EXK_EALIGN    (-2)  /* a pointer or stride breaks the 16-byte rule */
#define EXK_ETMAP     (-3)  /* cuTensorMapEncodeTiled rejected a tensor map */
#define EXK_EDRIVER   (-4)  /* the driver entry point could not be resolved */
#define EXK_EHEADS    (-5)  /* more than 16 query heads per KV head */
#define EXK_ESCRATCH  (-6)  /* partials larger than EXK_NOALLOC_SCRATCH_BYTES */

/* device status codes (written to the caller's int32 status word) */
#define EXK_S_OK             0
#define EXK_S_FULL_TIMEOUT   1  /* a consumer waited > 2 s for a staged page */
#define EXK_S_EMPTY_TIMEOUT  2  /* the TMA producer waited > 2 s for a free slot */
#define EXK_S_RAW_INDEX      3  /* rowoff/rowmask pointed past the raw pool */
#define EXK_S_CHAIN_TIMEOUT  4  /* (unused: the encoder no longer waits) */
#define EXK_S_DRAIN_TIMEOUT  5  /* in-flight TMA copies did not land within 2 s */
#define EXK_S_PEER_TIMEOUT   6  /* a peer merge waited > 2 s for another GPU's signal */
#define EXK_S_PAGE_INDEX     7  /* a block-table entry named a page outside the pool */

/* One compressed cache (keys or values of one layer): the six buffers of the
 * format above. raw_rows is the number of rows `raw` holds; indices at or
 * past it are reported (EXK_S_RAW_INDEX) and read as zero, never loaded. */
typedef struct exk_cview {
  const uint8_t *sm;
  const uint8_t *code;
  const uint8_t *base;
  const int32_t *rowmask;
  const int32_t *rowoff;
  const uint16_t *raw;
  int64_t raw_rows;
} exk_cview;

/* Split-K partials, laid out as the reference's workspace
 * (exactkv/kernels.py:290): o fp32 [rows, ns, 128] (unnormalised),
 * m fp32 [rows, ns] (running max of base-2 scores), l fp32 [rows, ns]
 * (sum of exp2(s - m)); rows = B * Hq. With the plan: ns splits of split_len
 * tokens, and `heads`, the KV heads one work item (one CTA at a time) covers:
 * 1, 2, 4 or 8 dividing Hkv, or 0 for the default (up to 8). The partials of
 * a split depend on `heads`, so calls that must agree bit for bit share it.
 * split_len = 0 selects a balanced plan (exk_plan_balanced): the whole call
 * only (splits [0, ns)), contiguous caches, host-side T or one device-side
 * length for the batch. */
typedef struct exk_partials {
  float *o;
  float *m;
  float *l;
  int32_t ns;
  int32_t split_len;
  int32_t heads;
} exk_partials;

/* Split plan: number of token splits per (sequence, KV head) and their length
 * (a multiple of 16), chosen so that B*Hkv*ns work items spread evenly over
 * `num_ctas` persistent CTAs (one per SM). Replaces choose_split()
 * (exactkv/kernels.py:273-277); the layout depends only on the arguments, so
 * the compressed and bf16 kernels and every GPU of a KV split share it. */
int exk_plan_splits(int B, int Hkv, int T, int num_ctas, int32_t *ns, int32_t *split_len);

/* Balanced plan for one whole call (the split kernel over every split, then
 * the merge) with host-side T: the (sequence, head group) stages of the call
 * are cut into num_ctas equal contiguous runs, one per CTA, across sequence
 * boundaries, so no CTA carries more work than another (with equal-length
 * splits, a batch whose work items do not fill whole waves leaves some CTAs
 * idle at the end). A unit's pieces are its splits; *ns receives the most
 * pieces any unit is cut into (use it with split_len = 0 in exk_partials), or
 * 0 when the uniform plan of exk_plan_splits is estimated faster. Replaces
 * choose_split() (exactkv/kernels.py:273-277) for whole calls; the bf16 and
 * compressed kernels given the same plan cut the work identically.
 * any_length != 0: the plan of a device-length call with one length for the
 * batch (exk_attention_*_devlen, T_stride 0) and capacity T; the kernel then
 * cuts the stages of the length it reads, and *ns is the bound
 * ceil(num_ctas / units) + 1 (units = B * head groups) that holds for every
 * length up to T. */
int exk_plan_balanced(int B, int Hkv, int T, int num_ctas, int consumer_warps, int any_length,
                      int32_t *ns);

/* Number of SMs of a device (the default `num_ctas`). */
int exk_num_sms(int device);

/* Split-K decode attention over the compressed cache, splits [s0, s1) of the
 * plan in `ws`. q: bf16 [B, Hq, 128] contiguous, Hq = G * Hkv, 1 <= G <= 16.
 * consumer_warps: 4 or 8. Replaces _split_c_kernel (exactkv/kernels.py:142-165). */
int exk_attn_split_compressed(const uint16_t *q, const exk_cview *k, const exk_cview *v,
                              int B, int TS, int Hkv, int Hq, int T, int s0, int s1,
                              const exk_partials *ws, int consumer_warps, float qk_scale,
                              int32_t *status, int device, void *stream);

/* The same computation on uncompressed bf16 K, V [B, TS, Hkv, 128]
 * (contiguous). Bit-identical to exk_attn_split_compressed on the same values,
 * plan and consumer_warps. Replaces _split_ref_kernel (exactkv/kernels.py:168-194). */
int exk_attn_split_bf16(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                        int B, int TS, int Hkv, int Hq, int T, int s0, int s1,
                        const exk_partials *ws, int consumer_warps, float qk_scale,
                        int32_t *status, int device, void *stream);

/* Merge of the split partials into bf16 out [rows, 128]:
 * out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M), M = max_s m_s.
 * Up to 16 splits: one warp per row, sums in split order. More: one CTA per
 * row, each warp folding chunks of 8 splits with its running maximum, the
 * warps combined in order; the order depends only on ns, so merges of the same
 * splits agree bit for bit. Replaces _reduce_kernel (exactkv/kernels.py:33-43). */
int exk_attn_merge(const exk_partials *ws, int rows, uint16_t *out, int device, void *stream);

/* Splits [s0, s1) of `ws` merged into one partial per row, the partial of the
 * union of those splits in the layout of a single split's: o [rows, 128]
 * (unnormalised), m [rows] (their maximum), l [rows]. A later merge combines
 * such partials like splits. The KV-sequence split reduces each GPU's run of
 * splits this way, so the GPUs exchange one partial per row each. No
 * counterpart in the reference. */
int exk_attn_merge_partial(const exk_partials *ws, int rows, int s0, int s1, float *o, float *m, float *l,
                           int device, void *stream);

/* Merge of split partials all-gathered from the `world` GPUs of a KV-sequence
 * split (world <= 16), straight from the gathered buffer: rank r's block (rows
 * * nmax * 130 floats rounded up to a multiple of 4, so each block starts
 * 16-byte aligned) holds o [rows, nmax, 128], then m and l [rows, nmax];
 * its first counts[r] (host array) columns are the next splits of the
 * sequence. Same arithmetic as exk_attn_merge over the splits in order, so a
 * split sequence gives the single-GPU result bit for bit. The reference has no
 * multi-GPU path; the merge itself replaces _reduce_kernel
 * (exactkv/kernels.py:33-43). */
int exk_attn_merge_gathered(const float *buf, int world, const int32_t *counts, int nmax, int rows,
                            uint16_t *out, int device, void *stream);

/* exk_attn_merge_gathered without the all-gather: blocks[r] (host array of
 * `world` device pointers, in this process's address space: this GPU's own
 * block and the peers' blocks mapped over NVLink, e.g. symmetric memory) is
 * rank r's block, read in place. `flags` (this GPU's uint32 [world], zeroed
 * before the first call) and peer_flags[p] (word `rank` of peer p's flags)
 * carry the exchange: every CTA first stores `epoch` into each peer's word
 * (system-scope release), then waits until flags[p] >= epoch for every peer
 * (acquire; at most 2 s, then EXK_S_PEER_TIMEOUT in *status and no output).
 * epoch counts the calls from 1, the same on every rank, and the caller
 * alternates two blocks per rank (the block of call e is rewritten at call
 * e + 2, after every peer finished reading it). Each rank's split kernel must
 * have written its block earlier on `stream`. No counterpart in the
 * reference. */
int exk_attn_merge_peers(const float *const *blocks, int world, int rank, const int32_t *counts, int nmax,
                         int rows, uint32_t *flags, uint32_t *const *peer_flags, uint32_t epoch,
                         uint16_t *out, int32_t *status, int device, void *stream);

/* One whole decode-attention call: every split of the plan in `ws`, then the
 * merge into bf16 out [B, Hq, 128] (exk_attn_merge), enqueued together; the
 * merge is a programmatic dependent launch, so its start overlaps the split
 * kernel's end. Replaces attention_compressed (exactkv/kernels.py:310-318):
 * the split kernel plus _reduce (exactkv/kernels.py:295-299). */
int exk_attention_compressed(const uint16_t *q, const exk_cview *k, const exk_cview *v,
                             int B, int TS, int Hkv, int Hq, int T, const exk_partials *ws,
                             uint16_t *out, int consumer_warps, float qk_scale,
                             int32_t *status, int device, void *stream);

/* exk_attention_compressed with the valid lengths read on the device: sequence
 * b holds T_b = min(T_cap, T_dev[b * T_stride] + T_add) tokens (T_stride 0: one
 * length for the batch; 1: one per sequence, a variable-length batch), so one
 * enqueued call (e.g. inside a captured CUDA graph) serves every step of a
 * growing cache. `ws` must hold the plan for T_cap (its splits exactly cover
 * T_cap); of that plan the kernel keeps the number of splits ns and cuts
 * sequence b into ns runs of ceil(ceil(T_b / 16) / ns) pages, so the work
 * stays balanced at any length (runs past T_b are empty and weigh nothing).
 * Same results as exk_attention_compressed with ns splits of that length at
 * length T_b (ns <= 256). With a balanced plan (split_len 0, from
 * exk_plan_balanced with any_length set; T_stride 0 only) the kernel cuts the
 * call's stages at the length it reads into one equal run per SM, as
 * exk_attention_compressed does for a host-side T. With advance != 0
 * (T_stride 0 only) the merge then adds `advance` to *T_dev (the end of a
 * step). No counterpart in the reference (its calls take one host-side T). */
int exk_attention_compressed_devlen(const uint16_t *q, const exk_cview *k, const exk_cview *v,
                                    int B, int TS, int Hkv, int Hq, int T_cap, int32_t *T_dev,
                                    int T_add, int T_stride, int advance, const exk_partials *ws,
                                    uint16_t *out, int consumer_warps, float qk_scale, int32_t *status,
                                    int device, void *stream);

/* The bf16 sibling of exk_attention_compressed_devlen (bit-identical on the same
 * values, plan, lengths and consumer_warps). */
int exk_attention_bf16_devlen(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                              int B, int TS, int Hkv, int Hq, int T_cap, int32_t *T_dev, int T_add,
                              int T_stride, int advance, const exk_partials *ws, uint16_t *out,
                              int consumer_warps, float qk_scale, int32_t *status, int device,
                              void *stream);

/* The bf16 sibling of exk_attention_compressed (bit-identical on the same values,
 * plan and consumer_warps). Replaces attention_reference (exactkv/kernels.py:321-328). */
int exk_attention_bf16(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                       int B, int TS, int Hkv, int Hq, int T, const exk_partials *ws,
                       uint16_t *out, int consumer_warps, float qk_scale,
                       int32_t *status, int device, void *stream);

/* Page encoder: encodes nb sequences x npg pages of `src` (bf16 bits, element
 * strides s_b, s_pg, s_p, s_h for sequence, page, token, head; channels
 * contiguous) into sequences b0.. and pages pg0.. of the buffers. Raw rows get
 * pool slots cnt, cnt+1, ... in (sequence, page, head) order — the order of
 * the reference's encode_reference; `cnt` advances even past raw_cap, but
 * slots at or past raw_cap are not written (the caller grows the pool and
 * encodes again). Four launches on `stream` (encode, chunk sums, chunk scan,
 * slot placement + raw copy).
 * Replaces _encode_pages_kernel/encode_pages (exactkv/kernels.py:233-268, 340-346). */
int exk_encode_pages(const uint16_t *src, int64_t s_b, int64_t s_pg, int64_t s_p, int64_t s_h,
                     uint8_t *sm, uint8_t *code, uint8_t *base, int32_t *rowmask, int32_t *rowoff,
                     uint16_t *raw, int64_t raw_cap, int32_t *cnt,
                     int b0, int pg0, int nb, int npg, int H, int TS,
                     int32_t *status, int device, void *stream);

/* One decode step's append with the length on the device (the whole step can
 * be enqueued once and replayed, e.g. in a CUDA graph). T_dev[b * T_stride] =
 * tokens sequence b holds before the step (T_stride 0: one length for the
 * batch; 1: a variable-length batch, each sequence on its own row and pages). Writes x [B, H, 128] (strides x_sb, x_sh; channels
 * contiguous) into row *T_dev % 16 of each (sequence, head)'s tail page — the
 * raw rows [raw_cap + (b*H + h)*16, +16) of the pool — and, when that fills
 * page (*T_dev + 1)/16 - 1, encodes the page exactly as exk_encode_pages does
 * (raw rows from slot *cnt, skipped at or past raw_cap) and opens the next
 * tail page (rowmask 0xFFFF, rowoff at its tail rows). Three launches; on
 * steps that fill no page the last two return at once. The caller keeps
 * raw_cap - *cnt at least B*H*16 rows ahead of the pages it will append.
 * Replaces the reference's append + encode_pages of a full tail page
 * (exactkv/cache.py:100-119) without its host synchronisation. */
int exk_append_token(const uint16_t *x, int64_t x_sb, int64_t x_sh, uint8_t *sm, uint8_t *code,
                     uint8_t *base, int32_t *rowmask, int32_t *rowoff, uint16_t *raw, int64_t raw_cap,
                     int32_t *cnt, int B, int H, int TS, const int32_t *T_dev, int T_stride,
                     int32_t *status, int device, void *stream);

/* Failure-detection self-test: one thread waits for an mbarrier phase that never
 * completes, with the kernels' own bounded wait shortened to limit_ns (at most
 * the kernels' 2 s), and writes EXK_S_FULL_TIMEOUT to *status when it gives up.
 * Nothing is in flight, so the context stays usable. No counterpart in the
 * reference. */
int exk_selftest_wait_timeout(int32_t *status, uint64_t limit_ns, int device, void *stream);

/* *T_dev += n on `stream` (the end of a device-length decode step). */
int exk_advance_length(int32_t *T_dev, int n, int device, void *stream);

/* Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from
 * page-locked host memory mapped into the device's address space (as
 * cudaHostAlloc gives it) into device memory, by a kernel on `stream` rather
 * than a copy-engine transfer: a decode step's inputs then reach the device
 * with no hand-off between the copy engine and the kernels before and after
 * them. EXK_EARG when either address is not reachable from the device. No
 * counterpart in the reference. */
int exk_copy_from_host(void *dst, const void *src, int64_t bytes, int device, void *stream);

/* Decode attention over paged caches: the cache buffers `k`, `v` are a pool of
 * pool_pages 16-token pages (sm [pool_pages * 16, Hkv, 128], code, base
 * [pool_pages, Hkv, 128], rowmask/rowoff [pool_pages, Hkv], raw as usual — any
 * [B', TS'] cache seen as B' * TS' / 16 pages), and page p of sequence b is
 * pool page block_table[b * max_pages + p] (int32 [B, max_pages], device).
 * seq_lens (int32 [B], device) holds each sequence's tokens (at most
 * max_pages * 16). `ws` holds the plan for max_pages * 16 tokens, used as in
 * exk_attention_compressed_devlen with one length per sequence; same results
 * as that call over the same pages laid out contiguously. The head group must
 * equal consumer_warps (Hkv a multiple of 8 with 8 warps, of 4 with 4), one
 * page per head per stage. An entry outside the pool reads as zeros and sets
 * EXK_S_PAGE_INDEX. No counterpart in the reference (its cache is one
 * contiguous [B, TS] block per layer). */
int exk_attention_compressed_paged(const uint16_t *q, const exk_cview *k, const exk_cview *v, int pool_pages,
                                   int Hkv, int B, int Hq, const int32_t *block_table, int max_pages,
                                   const int32_t *seq_lens, const exk_partials *ws, uint16_t *out,
                                   int consumer_warps, float qk_scale, int32_t *status, int device, void *stream);

/* The bf16 sibling of exk_attention_compressed_paged over bf16 pools
 * k, v [pool_pages * 16, Hkv, 128]; bit-identical for the same values. */
int exk_attention_bf16_paged(const uint16_t *q, const uint16_t *k, const uint16_t *v, int pool_pages, int Hkv,
                             int B, int Hq, const int32_t *block_table, int max_pages, const int32_t *seq_lens,
                             const exk_partials *ws, uint16_t *out, int consumer_warps, float qk_scale,
                             int32_t *status, int device, void *stream);

/* Compressed cache -> bf16 out [B, T, H, 128] through the attention kernel's
 * decoder. Replaces _dec_only_kernel/decode_to_bf16 (exactkv/kernels.py:197-211, 331-337). */
int exk_decode_to_bf16(const exk_cview *c, int B, int TS, int H, int T, uint16_t *out,
                       int32_t *status, int device, void *stream);

/* Split-K decode attention over the compressed cache that allocates nothing
 * and takes no workspace: the split partials live in a fixed device array of
 * EXK_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads the
 * library holds until the process exits. For callers that cannot allocate
 * device memory when they call (a runtime with a fixed memory plan, a plugin
 * whose enqueue must not call cudaMalloc). Same arguments and result as
 * exk_attn_split_compressed over the full plan followed by exk_attn_merge into
 * out [B*Hq, 128]. Returns EXK_ESCRATCH when B*Hq x splits x 130 fp32 exceed
 * the array (for example 32 sequences x 32 query heads at 4096 tokens: 1024
 * rows x 9 splits x 520 B = 4.79 MB is refused; 16 sequences fit). Shape
 * errors (EXK_EARG, EXK_EHEADS) and output errors are reported before the
 * size check, and nothing is launched when any argument is refused. The first call on a device looks up the array's device address
 * (make it before any stream capture). All calls on a GPU share the array:
 * calls that overlap on the GPU race. No counterpart in the reference. */
#define EXK_NOALLOC_SCRATCH_BYTES (4u << 20)
int exk_attention_compressed_noalloc(const uint16_t *q, const exk_cview *k, const exk_cview *v,
                                     int B, int TS, int Hkv, int Hq, int T, int consumer_warps,
                                     float qk_scale, uint16_t *out, int32_t *status, int device,
                                     void *stream);

/* Human-readable text for a return value or a device status code. */
const char *exk_error_string(int code);
const char *exk_status_string(int code);

#ifdef __cplusplus
}
#endif

#endif /* EXACTKV_B200_H */
