/*
 * aspida_attn.h — C ABI of libaspida_attn.so, the B200 (sm_100a) attention
 * library for the Aspida inference engine.
 *
 * The library is a drop-in for the attention part of Aspida's dlopen'd GPU
 * shim (libaspidagpu.so). Citations name the reference interface each entry
 * replaces, as path:line inside the reference project.
 *
 * Conventions
 *  - Every pointer marked "dev" is CUDA device memory; "host" is host memory.
 *  - KV layout is the shim's: fp16, row-major [max_len][nkv*hd], i.e.
 *    [pos][kv_head][dim], one row per position (gpu/gpu_matvec.cu:1312).
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).
 *  - Entry points returning int return 0 on success, a negative ASPIDA_ERR_*
 *    for argument/state errors, or a positive cudaError_t value. Every
 *    non-zero status is also latched for aspida_gpu_last_error().
 *  - No CPU fallback: a shape the kernels do not support is rejected with
 *    ASPIDA_ERR_UNSUPPORTED.
 *  - Calls on distinct streams may run concurrently; scratch memory is either
 *    caller-provided (workspace) or owned by the KV state / per stream.
 */
#ifndef ASPIDA_ATTN_H
#define ASPIDA_ATTN_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASPIDA_OK 0
#define ASPIDA_ERR_ARG (-1)         /* bad argument (sizes, null pointers)   */
#define ASPIDA_ERR_HANDLE (-2)      /* unknown or freed handle / slot        */
#define ASPIDA_ERR_NOMEM (-3)       /* device allocation failed              */
#define ASPIDA_ERR_UNSUPPORTED (-4) /* shape outside the kernels' coverage   */
#define ASPIDA_ERR_WORKSPACE (-5)   /* caller workspace smaller than needed  */
#define ASPIDA_ERR_DEVICE (-6)      /* a kernel's bounded wait ran out       */

/* ------------------------------------------------------------------------
 * KV-state lifecycle
 * ------------------------------------------------------------------------ */

/* Allocate a resident fp16 K/V cache of max_len rows x kvd halves each.
 * Returns a handle >= 0, or -1 on failure (bad sizes / allocation failure).
 * `nq` is accepted for signature compatibility; this library keeps no
 * per-head score scratch, so it only participates in argument checking.
 * Replaces aspida_gpu_fattn_new, gpu/gpu_matvec.cu:1316. */
int aspida_gpu_fattn_new(int max_len, int kvd, int nq);

/* Synchronise the device, then release the state; the handle is reused.
 * Unknown handles are ignored. Replaces gpu/gpu_matvec.cu:1335. */
void aspida_gpu_fattn_free(int handle);

/* Copy the first `rows` K/V rows of `handle` into a retained snapshot slot
 * (slot = -1 allocates a new one; an existing slot of the same rows/kvd is
 * overwritten in place). Returns the slot, or -1.
 * Replaces aspida_gpu_fattn_snapshot, gpu/gpu_matvec.cu:1359. */
int aspida_gpu_fattn_snapshot(int handle, int rows, int slot);

/* Copy snapshot `slot` back into rows 0..rows-1 of `handle`. Returns 0 or -1.
 * Replaces aspida_gpu_fattn_restore, gpu/gpu_matvec.cu:1391. */
int aspida_gpu_fattn_restore(int handle, int slot);

/* Free every retained snapshot. Replaces gpu/gpu_matvec.cu:1409. */
void aspida_gpu_prefix_reset(void);

/* Return and clear the first non-zero status latched since the last call
 * (or a pending CUDA error). 0 = no error.
 * Replaces aspida_gpu_last_error, gpu/gpu_matvec.cu:2348. */
int aspida_gpu_last_error(void);

/* Device pointers and geometry of a state (no counterpart in the shim, where
 * the state is only reachable inside the library; exported so a caller can
 * run the attention entry points below on handle-owned caches).
 * Returns 0 or ASPIDA_ERR_HANDLE. Any output pointer may be NULL. */
int aspida_gpu_fattn_kv(int handle, void** K, void** V, int* max_len, int* kvd);

/* Synchronise the current device and return (then clear) the device status
 * word that a kernel sets when one of its bounded waits runs out:
 * 0 = none, ASPIDA_ERR_DEVICE otherwise. The word is compiled into the
 * library (one per device), so no call allocates or synchronises to set it
 * up; every entry point, aspida_attn_decode_noalloc included, reports there. */
int aspida_attn_device_status(void);

/* Where the device status word was set (a code identifying the wait that
 * ran out: 10/11 decode producer/consumer, 60 the peer exchange's flag
 * wait; other values name mbarrier waits of the prefill kernel), or 0 if
 * it is clear. Does not synchronise or clear; call it before
 * aspida_attn_device_status(), after the work has finished. */
int aspida_attn_device_status_where(void);

/* Test hook: make the next `n` device allocations made by the library fail
 * (as cudaMalloc would on an exhausted device). n = 0 disarms it. */
void aspida_attn_debug_fail_allocs(int n);

/* ------------------------------------------------------------------------
 * Pre-attention step: per-head RMSNorm (optional), partial RoPE, and the
 * fp16 K/V append for P consecutive tokens at positions pos_start..+P-1.
 * Replaces k_fattn_prep / k_fattn_prep_chunk (gpu/gpu_matvec.cu:1449-1503,
 * 3235-3292) and the RoPE of LLM_RoPE.Apply_Sections (src/llm/llm_rope.adb:84).
 *   q      dev f32 [P][nq*hd]    raw query rows (gate already split off)
 *   k, v   dev f32 [P][nkv*hd]   raw key / value rows
 *   q_norm, k_norm  dev f32 [hd] RMSNorm weights, or NULL for no QK-norm
 *   q_out  dev [P][nq*hd], f32 (q_out_fp16 = 0) or fp16 (q_out_fp16 = 1)
 *   K, V   dev fp16 cache [max_len][nkv*hd]; rows pos_start..+P-1 written
 *   RoPE:  rd rotated dims (<= hd, even), base, freq_scale (PI), m_scale,
 *          yarn_on/corr_lo/corr_hi (YaRN ramp), ff dev [rd/2] (use_ff),
 *          interleaved (adjacent pairs) or NeoX split-half, sec_total:
 *          pairs i >= sec_total use position 0 (reference section quirk;
 *          pass rd/2 to rotate every pair).
 * ------------------------------------------------------------------------ */
int aspida_attn_prep(const float* q, const float* k, const float* v, int P, int nq, int nkv,
                     int hd, const float* q_norm, const float* k_norm, float eps, void* q_out,
                     int q_out_fp16, void* K, void* V, int max_len, int pos_start, int rd,
                     float base, float freq_scale, float m_scale, int yarn_on, float corr_lo,
                     float corr_hi, const float* ff, int use_ff, int interleaved, int sec_total,
                     void* stream);

/* Paged form of aspida_attn_prep: K_pool / V_pool are fp16 pools of blocks of
 * block_size rows ([blocks*block_size][nkv*hd]); the new rows go to
 * block_table[pos / block_size] * block_size + pos % block_size, the KV_Pool
 * block tables of src/llm/kv_pool.ads:1-47. pos == NULL: P tokens of one
 * sequence at pos_start.. through block_table [max_blocks]; pos != NULL
 * (dev i32 [P]): a decode batch, row t at pos[t] through block_table row t
 * ([P][max_blocks]). Positions must lie below max_blocks*block_size. */
int aspida_attn_prep_paged(const float* q, const float* k, const float* v, int P, int nq, int nkv,
                           int hd, const float* q_norm, const float* k_norm, float eps,
                           void* q_out, int q_out_fp16, void* K_pool, void* V_pool,
                           const int* block_table, int max_blocks, int block_size, int pos_start,
                           const int* pos, int rd, float base, float freq_scale, float m_scale,
                           int yarn_on, float corr_lo, float corr_hi, const float* ff,
                           int use_ff, int interleaved, int sec_total, void* stream);

/* ------------------------------------------------------------------------
 * Decode attention (one new token per sequence, GQA, split-KV).
 * Replaces the k_fattn_attend / k_fattn_attend_b launches
 * (gpu/gpu_matvec.cu:1507-1609, called at 2303-2304 and 2887-2892).
 *   q        dev f32 [B][nq*hd]  roped queries
 *   gate     dev f32 [B][nq*hd]  or NULL; out *= sigmoid(gate) (Qwen gate)
 *   K, V     dev tables [B] of dev fp16 caches [rows][nkv*hd]
 *   pos      dev i32 [B]  0-based position of the new token: keys 0..pos
 *   max_len  dev i32 [B]  or NULL: keys are clamped below max_len[b]
 *   out      dev f32 [B][nq*hd]
 *   scale    softmax scale (1/sqrt(hd) for Llama/Qwen, 1.0 for Gemma)
 *   window   sliding window (keys max(0,pos-window+1)..pos), 0 = none
 *   softcap  s <- softcap*tanh(s/softcap) after scaling, 0 = none
 *   max_kv_len  upper bound of pos+1 over the batch (sizes the grid)
 *   chunk    0 = automatic (one contiguous range of keys per resident warp);
 *            > 0 = at least `chunk` keys per warp range (fewer, longer ranges)
 *   workspace/workspace_bytes  dev scratch (256-byte aligned) of at least
 *            aspida_attn_decode_workspace_size bytes: (m, l, o) partials of
 *            sequences split between CTAs and the unit offsets. No
 *            initialisation is needed. Calls that share a workspace must not
 *            overlap on the GPU.
 * Supported: hd in {64,128,256}, nq % nkv == 0, nq/nkv <= 8.
 * ------------------------------------------------------------------------ */
size_t aspida_attn_decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len,
                                         int chunk);
int aspida_attn_decode(const float* q, const float* gate, const void* const* K,
                       const void* const* V, const int* pos, const int* max_len, float* out,
                       int B, int nq, int nkv, int hd, float scale, int window, float softcap,
                       int max_kv_len, int chunk, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Paged-KV decode: the K and V rows of all sequences live in shared pools of
 * fixed-size blocks, dev fp16 [num_blocks * block_size][nkv*hd] (block k =
 * rows k*block_size..); row `key` of sequence b is pool row
 * block_table[b*max_blocks + key/block_size]*block_size + key%block_size.
 * Blocks may be shared between sequences (prefix sharing). Arguments as for
 * aspida_attn_decode otherwise (max_kv_len <= max_blocks*block_size). The
 * block-table model follows KV_Pool (src/llm/kv_pool.ads:1-47), which the
 * reference keeps on the host only. */
int aspida_attn_decode_paged(const float* q, const float* gate, const void* K_pool,
                             const void* V_pool, const int* block_table, int max_blocks,
                             int block_size, const int* pos, float* out, int B, int nq, int nkv,
                             int hd, float scale, int window, float softcap, int max_kv_len,
                             int chunk, void* workspace, size_t workspace_bytes, void* stream);

/* Split-KV partial for sequence-parallel decode: attend keys
 * kv_lo[b]..kv_hi[b]-1 of each cache and write the unnormalised partial
 * (m = running max in natural-log units, l = sum of exp(s-m), o = sum of
 * exp(s-m)*v) per (sequence, head): m, l dev f32 [B][nq]; o dev f32 [B][nq][hd].
 * An empty range gives m = -3.4e38, l = 0, o = 0. This is the per-slice half
 * of flash-decoding split-K (k_splitk, gpu/fattn_sk.cu:38-83), extended to a
 * slice per GPU. */
int aspida_attn_decode_partial(const float* q, const void* const* K, const void* const* V,
                               const int* kv_lo, const int* kv_hi, float* m, float* l, float* o,
                               int B, int nq, int nkv, int hd, float scale, float softcap,
                               int max_kv_len, int chunk, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Decode fused with the pre-attention step (the row-per-sequence case of
 * k_fattn_prep, gpu/gpu_matvec.cu:1449-1503, followed by the attention of
 * k_fattn_attend_b): q_raw dev f32 [B][nq*hd] un-normed, un-rotated queries;
 * k_raw, v_raw dev f32 [B][nkv*hd] the new token's key / value rows, appended
 * at pos[b] (K RMSNorm'ed with k_norm if given and rotated, V as given, both
 * fp16) unless pos[b] >= max_len[b]; queries RMSNorm'ed with q_norm if given
 * and rotated in registers. RoPE parameters as for aspida_attn_prep (NeoX
 * requires rd % 32 == 0, else ASPIDA_ERR_UNSUPPORTED); the cache rows written
 * equal aspida_attn_prep's. Other arguments and the workspace as
 * aspida_attn_decode (fp16 per-sequence caches). One launch replaces
 * aspida_attn_prep + aspida_attn_decode; measured on B200 at config 2 it is
 * slower than the two (0.137 vs ~0.107 ms): the rotation and the appends
 * serialise on the bandwidth-bound kernel's critical path, where the prep
 * kernel spreads them over the whole GPU. */
int aspida_attn_decode_fused(const float* q_raw, const float* k_raw, const float* v_raw,
                             const float* gate, const void* const* K, const void* const* V,
                             const int* pos, const int* max_len, float* out, int B, int nq,
                             int nkv, int hd, const float* q_norm, const float* k_norm, float eps,
                             int rd, float base, float freq_scale, float m_scale, int yarn_on,
                             float corr_lo, float corr_hi, const float* ff, int use_ff,
                             int interleaved, int sec_total, float scale, int window,
                             float softcap, int max_kv_len, int chunk, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Decode over Q8_0 KV caches: the storage of the reference's KVMODE 2
 * (k_gqa_kv<..., 2>, gpu/fattn_kvhalf.cu:55-130; tile-load dequant at 88-92):
 *   K8, V8          dev tables [B] of dev int8 caches [rows][nkv*hd]
 *   K_scales, V_scales  dev tables [B] of dev fp16 scales [rows][nkv*hd/32],
 *                   one per 32-value block along a row; value = int8 * scale
 * Other arguments and the workspace as aspida_attn_decode. Caches 16-byte
 * aligned. Supported: hd in {64, 128, 256} with nkv*hd >= 256 (a group of
 * kv heads whose scales fill 16-byte units); else ASPIDA_ERR_UNSUPPORTED. */
int aspida_attn_decode_q8(const float* q, const float* gate, const void* const* K8,
                          const void* const* V8, const void* const* K_scales,
                          const void* const* V_scales, const int* pos, const int* max_len,
                          float* out, int B, int nq, int nkv, int hd, float scale, int window,
                          float softcap, int max_kv_len, int chunk, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Decode over fp8 (e4m3) KV caches, the fp8 half of the 8-bit KV modes
 * (the reference's 8-bit mode is Q8_0, gpu/fattn_kvhalf.cu:55-152; fp8 has no
 * counterpart there). Same storage geometry and table convention as
 * aspida_attn_decode_q8: K8 / V8 tables of uint8 e4m3 code caches
 * [rows][nkv*hd], K_scales / V_scales tables of fp16 scales [rows][nkv*hd/32]
 * (one per 32-value block along a row); value = e4m3(code) * scale, which
 * aspida_attn_quantize_fp8 writes. Other arguments, the workspace and the
 * supported shapes as aspida_attn_decode_q8. */
int aspida_attn_decode_fp8(const float* q, const float* gate, const void* const* K8,
                           const void* const* V8, const void* const* K_scales,
                           const void* const* V_scales, const int* pos, const int* max_len,
                           float* out, int B, int nq, int nkv, int hd, float scale, int window,
                           float softcap, int max_kv_len, int chunk, void* workspace,
                           size_t workspace_bytes, void* stream);

/* fp8 (e4m3) quantiser for aspida_attn_decode_fp8's caches: nblk blocks of 32
 * consecutive f32 values; scales[b] = fp16(max|v| / 448); code =
 * e4m3(v / float(scales[b])), round to nearest even, saturating at +-448;
 * a block with scale 0 gets zeros. in and q 16-byte aligned. */
int aspida_attn_quantize_fp8(const float* in, void* q, void* scales, long long nblk,
                             void* stream);

/* Gated causal prefill over Q8_0 caches with the argument meaning of the
 * reference's k_gqa_kv<..., 2> (gpu/fattn_kvhalf.cu:59-130, launched at
 * 162-190): q_all / gate f32 [P][nq*hd] (q 16-byte aligned), K8 / V8 int8
 * caches and K_scales / V_scales fp16 scales (Q8_0 layout, >= pos_start+P
 * rows), out f32 [P][nq*hd]; query t at position pos_start+t attends keys
 * 0..pos_start+t, scale 1/sqrt(hd), out *= sigmoid(gate). The cache prefix
 * is dequantised into per-stream fp16 scratch (int8 x scale, rounded to fp16)
 * and the tcgen05 prefill runs on it. Zeroes `out` on failure. */
int aspida_attn_prefill_q8_gated(const float* q_all, const float* gate, const void* K8,
                                 const void* V8, const void* K_scales, const void* V_scales,
                                 float* out, int nq, int nkv, int hd, int P, int pos_start,
                                 void* stream);

/* Q8_0 quantiser, the algorithm of k_to_q8 (gpu/fattn_kvhalf.cu:143-152):
 * nblk blocks of 32 consecutive f32 values; scales[b] = fp16(max|v|/127),
 * q = clamp(round-to-nearest-even(v * (1/d)), -127, 127), zeros for an
 * all-zero block. Appending rows to a Q8_0 cache is this call on the rows'
 * f32 values (nblk = rows*nkv*hd/32) with q/scales pointing at the rows.
 * in and q 16-byte aligned. */
int aspida_attn_quantize_q8(const float* in, void* q, void* scales, long long nblk,
                            void* stream);

/* Log-sum-exp merge of S partials (k_combine, gpu/fattn_sk.cu:84-97):
 *   m, l dev f32 [S][rows]; o dev f32 [S][rows][hd]; gate dev f32 [rows][hd]
 *   or NULL; out dev f32 [rows][hd] = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s. */
int aspida_attn_merge(const float* m, const float* l, const float* o, const float* gate,
                      float* out, int S, int rows, int hd, void* stream);

/* Same merge over partials gathered per rank into one buffer: partial s of
 * m, l and o starts part_stride floats after partial s-1 (e.g. each rank's
 * packed [m | l | o] block of an all-gather). No counterpart in the
 * reference; the strided form spares a copy after the exchange. */
int aspida_attn_merge_strided(const float* m, const float* l, const float* o, const float* gate,
                              float* out, int S, int rows, int hd, long part_stride,
                              void* stream);

/* ------------------------------------------------------------------------
 * NVLink peer exchange for sequence-parallel decode, fused with the merge.
 * No counterpart in the reference (it has no multi-GPU inference); it
 * replaces an NCCL all-gather of the packed partials + aspida_attn_merge.
 *   aspida_attn_peer_buffer_size(world, rows, hd): bytes of one rank's
 *     receive buffer (two step-parity banks of `world` partial slots + flags).
 *   aspida_attn_peer_alloc: cudaMalloc + zero-fill that many bytes and write
 *     its 64-byte CUDA IPC handle (cudaIpcMemHandle_t) to ipc_handle.
 *   aspida_attn_peer_open / _close: map / unmap another rank's buffer from
 *     its handle (same node, peer access); _free releases one's own.
 *   aspida_attn_exchange_merge: `part` = this rank's packed partial
 *     [m[rows] | l[rows] | o[rows][hd]] (f32, 16-byte aligned, m in natural
 *     log units as aspida_attn_decode_partial writes it); recv = host array
 *     [world] of every rank's buffer as mapped in this process (recv[rank] =
 *     its own); step = 1, 2, 3, ... identical on every rank. Sends `part` to
 *     every rank over NVLink, waits (bounded) for every rank's partial of
 *     this step and writes the merged out[rows][hd] (x sigmoid(gate) if
 *     given). All ranks must call it once per step, in the same order, one
 *     rank per GPU. world <= 8. A rank that never arrives makes the wait run
 *     out after seconds: the device status word is set. */
size_t aspida_attn_peer_buffer_size(int world, int rows, int hd);
int aspida_attn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int aspida_attn_peer_open(const void* ipc_handle, void** peer_ptr);
int aspida_attn_peer_close(void* peer_ptr);
int aspida_attn_peer_free(void* ptr);
int aspida_attn_exchange_merge(const float* part, void* const* recv, int world, int rank,
                               unsigned long long step, const float* gate, float* out, int rows,
                               int hd, void* stream);

/* aspida_attn_exchange_merge with two more arguments (no counterpart in the
 * reference):
 *   fail_word   int the kernel sets to a non-zero code when its wait runs
 *               out, besides the device status word; NULL = none. Pinned
 *               host memory (device-visible) lets the host see a failed
 *               exchange without synchronising the stream.
 *   wait_limit  flag polls per rank before the wait gives up (0 = the
 *               default of ~4M polls with backoff, seconds); a short limit
 *               lets a test make the wait run out quickly.
 * When the wait runs out the kernel writes no output and returns; the
 * exchange's two-bank reuse guarantee is then void, so the caller must not
 * run further steps on these buffers. */
int aspida_attn_exchange_merge_ex(const float* part, void* const* recv, int world, int rank,
                                  unsigned long long step, const float* gate, float* out,
                                  int rows, int hd, int* fail_word, long long wait_limit,
                                  void* stream);

/* ------------------------------------------------------------------------
 * Causal prefill attention on the tcgen05 tensor cores.
 * Replaces aspida_ggml_fattn_prefill (gpu/fattn_ggml.cuh:109-141) and the
 * shim's own prefill kernels (gpu/gpu_matvec.cu:3309-3682).
 *   q      dev fp16 [P][nq*hd]   roped queries (aspida_attn_prep, q_out_fp16)
 *   K, V   dev fp16 caches with >= pos_start+P rows of nkv*hd halves
 *   gate   dev f32 [P][nq*hd] or NULL (out *= sigmoid(gate))
 *   out    dev [P][nq*hd], fp16 (out_f32 = 0) or f32 (out_f32 = 1)
 *   query t (position pos_start+t) attends keys max(0, pos-window+1)..pos;
 *   scale / window / softcap as for decode.
 * All pointers 16-byte aligned. Supported: hd in {64, 128, 256}.
 * At hd 256, a chunk whose (query tile, head) items cannot fill the GPU has
 * each tile's key range split over CTAs; the partials live in library
 * scratch kept per (device, stream), allocated on first need. */
int aspida_attn_prefill(const void* q, const void* K, const void* V, const float* gate, void* out,
                        int out_f32, int nq, int nkv, int hd, int P, int pos_start, float scale,
                        int window, float softcap, void* stream);

/* Paged form of aspida_attn_prefill: K_pool / V_pool hold num_blocks blocks
 * of block_size rows; key row r of the sequence lives in pool row
 * block_table[r / block_size] * block_size + r % block_size (dev i32 table).
 * block_size must be a multiple of the kernel's key tile (128 for hd <= 128,
 * 64 for hd 256), else ASPIDA_ERR_UNSUPPORTED. Rows of the last block past
 * pos_start + P are read (with zero weight), so they must hold finite values
 * (a zero-initialised pool does). */
int aspida_attn_prefill_paged(const void* q, const void* K_pool, const void* V_pool,
                              const int* block_table, int num_blocks, int block_size,
                              const float* gate, void* out, int out_f32, int nq, int nkv, int hd,
                              int P, int pos_start, float scale, int window, float softcap,
                              void* stream);

/* Batched form: nseq sequences, each with its own q/K/V/gate/out pointers
 * and P / pos_start (host arrays of device pointers and host ints). */
int aspida_attn_prefill_batch(int nseq, const void* const* q, const void* const* K,
                              const void* const* V, const float* const* gate, void* const* out,
                              const int* P, const int* pos_start, int out_f32, int nq, int nkv,
                              int hd, float scale, int window, float softcap, void* stream);

/* Qwen gated prefill with the argument list of the shim's internal swap
 * point aspida_ggml_fattn_prefill (gpu/fattn_ggml.cuh:109-112), which it
 * replaces: q_all dev f32 [P][nq*hd] (prepped, 16-byte aligned), K/V dev
 * fp16 cache [>= pos_start+P][nkv*hd], gate dev f32 [P][nq*hd] or NULL,
 * out dev f32 [P][nq*hd]; scale 1/sqrt(hd); causal. Returns 0 (the shim's
 * `true`) or an error, in which case `out` is zeroed as the shim does. */
int aspida_attn_prefill_gated(const float* q_all, const void* K, const void* V, const float* gate,
                              float* out, int nq, int nkv, int hd, int P, int pos_start,
                              void* stream);

/* Host-buffer decode step for B resident states — the attention half of
 * aspida_gpu_fattn_step / chain_forward_batch (gpu/gpu_matvec.cu:1613, 2783)
 * without the projections: copies q/k/v/pos from host, runs prep (RoPE, no
 * QK-norm, KV append at pos[b]) and decode, copies the output to host and
 * synchronises the stream.
 *   handles host [B]; q host f32 [B][nq*hd]; k, v host f32 [B][nkv*hd];
 *   pos host [B]; out host f32 [B][nq*hd]. RoPE: NeoX or interleaved over
 *   rd dims with base (rd = 0 disables RoPE). */
int aspida_attn_step_host(const int* handles, int B, const float* q, const float* k,
                          const float* v, const int* pos, float* out, int nq, int nkv, int hd,
                          float scale, int window, float softcap, int rd, float base,
                          int interleaved, void* stream);

/* Allocation-free variant of aspida_attn_decode, for callers that cannot
 * allocate device memory (inside an allocator callback, under a budget
 * reserved up front, or on a thread that must not block on the device-wide
 * synchronisation cudaMalloc/cudaFree can imply). No counterpart in the
 * reference. Same arguments as aspida_attn_decode without the workspace:
 * its scratch is a 16 MiB array compiled into the library, held on every GPU
 * that loads it until exit. Returns ASPIDA_ERR_WORKSPACE when
 * aspida_attn_decode_workspace_size of the call exceeds that (e.g. B > ~360
 * at nkv 8, hd 128). The first call on each device looks up the array's
 * device address; make it before any stream capture. All calls share the
 * array, so calls that overlap on the GPU race: serialise them. A bounded
 * wait that runs out is reported by aspida_attn_device_status(), as for the
 * other entry points. */
int aspida_attn_decode_noalloc(const float* q, const float* gate, const void* const* K,
                               const void* const* V, const int* pos, const int* max_len,
                               float* out, int B, int nq, int nkv, int hd, float scale,
                               int window, float softcap, int max_kv_len, int chunk,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ASPIDA_ATTN_H */
