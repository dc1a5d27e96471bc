/*
 * nibblegemm_b200 -- C ABI of the B200 (sm_100a) W4A16 kernel library.
 *
 * Packed format (identical to arvindcr4/nibblegemm, python/nibblegemm/quant.py:8-54):
 *   qweight  int32 [K/8, N]: eight 4-bit codes along K per word, logical k of
 *            the word stored in nibble slot (k odd ? 4 + k/2 : k/2), i.e. slot
 *            order 0,4,1,5,2,6,3,7; code u means (u - 8) * scale.
 *   scales   fp16  [K/G, N]: one scale per (group of G rows of K, column).
 *   x        fp16 or bf16 [M, K] row-major;  y same dtype as x, [M, N].
 *   Y = X @ W with W[k, n] = (u[k, n] - 8) * scales[k / G, n].
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers, caller-owned, contiguous row-major.
 *     The library allocates nothing and never synchronises (except
 *     ng_device_status); work is enqueued on `stream` (a cudaStream_t;
 *     NULL = legacy default stream) of the current device.
 *   - Return value: NG_OK (0) or a positive NG_ERR_* status; nothing aborts.
 *     ng_status_string() names the status.  Validation happens before any
 *     launch, so a non-zero status from validation enqueues nothing.
 *   - Calls are thread-safe; the only library state is a per-device cache of
 *     device properties and kernel attributes, initialised on first use, and
 *     a per-device error word that kernels set when a bounded wait expires.
 */
#ifndef NIBBLEGEMM_B200_H
#define NIBBLEGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define NG_OK 0
#define NG_ERR_NULL_POINTER 1       /* a required pointer is NULL                     */
#define NG_ERR_BAD_DTYPE 2          /* dtype code not NG_DTYPE_F16 / NG_DTYPE_BF16     */
#define NG_ERR_BAD_SHAPE 3          /* M, K, N or group size inconsistent/unsupported  */
#define NG_ERR_MISALIGNED 4         /* a pointer lacks the alignment its loads need    */
#define NG_ERR_BAD_ARGUMENT 5       /* an option (splits, threads, algo, tile) out of range */
#define NG_ERR_LAUNCH 6             /* the CUDA launch itself failed                   */
#define NG_ERR_UNSUPPORTED_DEVICE 7 /* current device is not sm_100                    */
#define NG_ERR_CUDA 8               /* another CUDA runtime/driver call failed         */
#define NG_ERR_DEVICE_TIMEOUT 9     /* a kernel's bounded pipeline wait expired        */
#define NG_ERR_BAD_INDEX 10         /* a kernel met an index (token id) outside its table */

/* Activation / output element types. */
#define NG_DTYPE_F16 0
#define NG_DTYPE_BF16 1

/* Library ABI version (bumped on any signature change). */
int ng_abi_version(void);

/* Human-readable name of a status code (static storage, never NULL). */
const char* ng_status_string(int status);

/*
 * Synchronise `stream`, then return NG_ERR_DEVICE_TIMEOUT if any kernel of this
 * library on the current device gave up on a bounded wait since the last call,
 * else NG_ERR_BAD_INDEX if one met an out-of-range index (and clear both flags), NG_ERR_CUDA if the stream reports an error, else NG_OK.
 * No counterpart in the reference (its kernels have no waits that can expire).
 */
int ng_device_status(void* stream);

/*
 * Dense dequantisation: out[K, N] = (u - 8) * scale, one rounding to out_dtype.
 * Replaces the reference's `dequant_w4(Wq, S, group_size, fast)`
 * (csrc/dequant_kernel.cu:48-74, bound at csrc/bindings.cpp:19-20).
 *   fast != 0 : lop3 / magic-number decode;  fast == 0 : shift-mask-convert decode.
 *   Both are bit-exact with the CPU oracle for NG_DTYPE_F16 (the reference's
 *   only output type); NG_DTYPE_BF16 rounds the same exact product to bf16.
 *   Requires K % 8 == 0, K % group_size == 0, group_size % 8 == 0, N >= 1.
 */
int ng_dequant_w4(const int32_t* qweight, const uint16_t* scales, void* out, int out_dtype,
                  int K, int N, int group_size, int fast, void* stream);

/*
 * Decode-regime fused dequant GEMV, one launch.
 * Replaces the reference's `gemv_w4a16(X, Wq, S, group_size, version,
 * splits_override, threads_override)` (csrc/gemv_w4a16.cu:341-425, bound at
 * csrc/bindings.cpp:12-15), which takes its split-K workspace from the torch
 * caching allocator on every call; this one takes it from the caller.
 *   M in [1, 16]; N % 4 == 0; group_size in {64, 128, 256}; K % group_size == 0.
 *   Schedules:
 *   - tensor pipe (algo 3; needs the workspace): packed words decoded to magic-number fp16/bf16
 *     operands of mma.sync, fp32 accumulation; persistent CTAs with equal
 *     shares of (64-column tile, 128-value K slice) units; tiles split between
 *     CTAs are finished by the last CTA to arrive, summing in CTA order
 *     (deterministic).  `workspace`: ng_gemv_workspace_bytes(M, N) bytes,
 *     256-byte aligned, zero-filled before first use; its layout does not
 *     depend on M or N and each call leaves the part that must start at zero
 *     (per-tile arrival counters) at zero.  Calls sharing a workspace must not
 *     overlap on the GPU (one workspace per stream).
 *   - CUDA-core cluster split-K (algo 1 / 2; the workspace is
 *     not used): `splits` K slices (1..16, 0 = heuristic,
 *     raised if needed so a slice's activations fit on chip) reduced through
 *     distributed shared memory inside a thread-block cluster, fixed rank
 *     order; block_threads 0 (256), 128 or 256;  algo 1 = fp16 decode with
 *     packed-half2 FMA windows of 32 values flushed to fp32 (fp16 x only),
 *     algo 2 = fp32 decode with packed fp32x2 FMA (the default for bf16 x).
 *   - algo 0 (default), with block_threads == 0 and splits <= 8:
 *     algo 5 with one K slice per column tile when N >= 12288, M <= 8 and
 *     (M >= 2 or K <= 4096); algo 5 (stream-K) when M is 3..4 and the packed weight is
 *     >= 12 MiB; algo 5 when M > 4; otherwise algo 1 (fp16 x) / 2 (bf16 x).
 *   - bulk-copy ring (algo 4: M <= 8, algo 5: M <= 16; the workspace only for
 *     stream-K):
 *     one producer warp per CTA streams the CTA's (128-column, K-slice) weight
 *     block into a shared-memory ring with 2-D TMA loads, consumer warps
 *     decode from shared memory -- algo 4 with the algo 1 (fp16 x) / algo 2
 *     (bf16 x) arithmetic, algo 5 on the tensor pipe (magic-number operands to
 *     mma.sync, fp32 accumulation, offsets removed by a correction MMA);
 *     `splits` 1..8 = K slices reduced in a cluster as above; 0 = algo 5 on
 *     M <= 4 with K % 128 == 0 and a workspace: one CTA per SM with equal
 *     shares of 16-row blocks, split tiles finished through the workspace in
 *     fixed order -- "head/tail" when the column tiles fill half the SMs or
 *     more (tile CTAs stream each tile's first blocks, helper CTAs the rest),
 *     stream-K over the tile-major block list otherwise (measured slower than
 *     the clustered grid in a chain of launches where that grid leaves SMs
 *     free, so the default uses these only for M = 3..4 on long K); a
 *     heuristic K split when those do not apply.
 *   All are launched with programmatic stream serialisation: they start
 *   streaming their read-only weights while the previous kernel on the stream
 *   finishes, and read x / write y / touch the workspace only after it has.
 *   x, qweight 16-byte aligned; scales 8-byte aligned.
 */
int ng_gemv_w4a16(const void* x, int x_dtype, const int32_t* qweight, const uint16_t* scales,
                  void* y, int M, int K, int N, int group_size, int splits, int block_threads,
                  int algo, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Workspace bytes ng_gemv_w4a16 needs for an N-column weight on the current
 * device, every schedule included (0 if M or N is out of range).  No counterpart in the
 * reference, which allocates its workspace inside each call.
 */
size_t ng_gemv_workspace_bytes(int M, int N);

/*
 * Allocation-free variant of the tensor-pipe GEMV (ng_gemv_w4a16, algo 3).
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory at the point of the call (code inside an allocator or memory
 * hook, plugins whose host owns all allocation, allocation-free inference
 * loops) and so cannot supply a workspace.  The scratch space comes from a
 * fixed 3 MiB array in the library's device data, present on every GPU that
 * loads the library until the process exits.
 *   Same arguments and limits as ng_gemv_w4a16 otherwise; returns
 *   NG_ERR_BAD_SHAPE when the shape needs more scratch than the array holds
 *   (about N > 8 million columns on a 148-SM B200).
 *   The first call on a device looks up the array's device address (with that
 *   device current); make that first call before any stream capture.
 *   Each call clears the array's arrival counters on `stream` before the
 *   kernel (cudaMemsetAsync; nothing is allocated).  All calls on a device
 *   share the one array: calls that overlap on the GPU (different streams,
 *   concurrent graphs) race and must be serialised by the caller.
 */
int ng_gemv_w4a16_noalloc(const void* x, int x_dtype, const int32_t* qweight,
                          const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                          void* stream);

/*
 * Prefill-regime fused dequant GEMM on the sm_100 tensor cores: tcgen05.mma
 * with accumulators in tensor memory, activations staged by TMA, weight tiles
 * decoded by CUDA-core warps straight into the tensor cores' shared-memory
 * layout.  Persistent, warp-specialised, one launch.
 * Replaces the reference's `gemm_w4a16(X, Wq, S, group_size, version)`
 * (csrc/gemm_w4a16.cu:379-429, bound at csrc/bindings.cpp:16-18).
 *   Any M >= 1; K % 64 == 0; N % 4 == 0; group_size in {64, 128, 256};
 *   x, qweight 16-byte aligned; scales 2-byte aligned.
 *   tile_tokens: 0 = heuristic, else 16, 32, 64, 128, 192, 224, 240 or 256 rows
 *   of X per tile.
 *   workspace (may be NULL): ng_gemm_workspace_bytes(M, N) bytes, 256-byte
 *   aligned, zero-filled before first use.  With it, grids that would leave
 *   SMs idle (few tiles: small M, or N = 4096 with long K) are split along K;
 *   each split writes fp32 partials there and the last split of a tile to
 *   finish sums them in split order (deterministic) and re-arms the tile's
 *   counter, so the workspace is reusable as is.  Without it, no K split.
 *   Calls sharing a workspace must not overlap on the GPU.
 */
int ng_gemm_w4a16(const void* x, int x_dtype, const int32_t* qweight, const uint16_t* scales,
                  void* y, int M, int K, int N, int group_size, int tile_tokens, void* workspace,
                  size_t workspace_bytes, void* stream);
/* Workspace bytes ng_gemm_w4a16 can use for an [M, N] output on the current
 * device (0 if M or N is out of range). */
size_t ng_gemm_workspace_bytes(int M, int N);

/*
 * Tensor-parallel reduction for the decode step: one-shot all-reduce (sum) of
 * a small fp16/bf16 vector across the `world` GPUs of one node over NVLink
 * peer memory.  No counterpart in the reference (single-GPU); replaces the
 * NCCL all-reduce after each row-parallel projection.
 *   Set-up (once per communicator): every rank allocates its exchange buffer
 *   of ng_allreduce_buffer_bytes(world, max_elems) bytes with ng_ipc_alloc
 *   (zero-filled, exported as a 64-byte CUDA IPC handle) and a zero-filled
 *   array of 16 uint32 call counters (`epochs`), passes the handle to its
 *   peers, and maps the peers' buffers with ng_ipc_open.  `peer_buffers[p]` is rank p's buffer as mapped in this
 *   process (this rank's own buffer at index `rank`).
 *   Each call: every rank calls with the same n (<= max_elems) in the same
 *   order; `data` is reduced in place; the sum is taken in fp32 in rank order
 *   (every rank gets bit-identical results).  The kernel waits (bounded) for
 *   the peers' arrivals; a timeout is reported by ng_device_status.
 */
size_t ng_allreduce_buffer_bytes(int world, size_t max_elems);
int ng_allreduce_sum(void* data, int dtype, size_t n, void* const* peer_buffers, int rank,
                     int world, size_t max_elems, unsigned int* epochs, void* stream);
/* Allocate a zero-filled buffer on the current device and write its 64-byte
 * IPC handle to `handle` / free it.  Map a peer's buffer from its handle /
 * unmap it. */
int ng_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
int ng_ipc_free(void* dev_ptr);
int ng_ipc_open(const void* handle, void** dev_ptr);
int ng_ipc_close(void* dev_ptr);

/*
 * Decode-step kernels around the projections (no counterpart in the reference,
 * whose decode step is projections only; bench/bench_model.py:57-86).  All
 * take fp16 or bf16 activations (`dtype`), compute in fp32, enqueue on
 * `stream` and allocate nothing.
 *   ng_rmsnorm: per token h = x + residual (residual may be NULL; else h is
 *     written back to it), y = h * rsqrt(mean(h^2) + eps) * weight.  [M, H],
 *     H <= 8192.
 *   ng_rope_append: qkv [M, (Hq + 2 Hkv) * D] -> q_out [M, Hq, D] with RoPE
 *     ("rotate half" pairs (i, i + D/2), angle pos * theta^(-2i/D)), K rows
 *     rotated and V rows copied into k_cache / v_cache [M, max_ctx, Hkv, D]
 *     (one cache per sequence) at row pos[m] (device int array of M positions; rows outside [0, max_ctx)
 *     are not written).
 *   ng_attn_decode: GQA attention of q [M, Hq, D] (D = 128) over the first
 *     min(ctx_len[m], max_ctx) cache rows (device int array), softmax scale; the
 *     context is split in `splits` chunks whose fp32 partials
 *     (ng_attn_workspace_bytes) are combined in chunk order -> out [M, Hq, D].
 *   ng_silu_mul: gate_up [M, 2I] (gate | up) -> out [M, I] = silu(gate) * up.
 */
int ng_rmsnorm(const void* x, void* residual, const void* weight, void* y, int dtype, int M, int H,
               float eps, void* stream);
int ng_rope_append(const void* qkv, void* q_out, void* k_cache, void* v_cache, const int* pos,
                   int dtype, int M, int Hq, int Hkv, int D, float theta, int max_ctx,
                   void* stream);
/* Prefill of B sequences of S prompt tokens each (token m = b * S + s of the
 * [B * S, ...] activations, at position pos[b] + s; pos: device int array of B
 * start positions).  No counterpart in the reference, which benchmarks the
 * projections of a step only (bench/bench_model.py:43-86); these carry
 * BASELINE config 5's 2048-token prefill around ng_gemm_w4a16.
 *   ng_rope_prefill: ng_rope_append for runs of S consecutive positions per
 *     sequence: q_out [B * S, Hq, D], K / V rows into the caches at pos[b] + s.
 *   ng_attn_prefill: causal GQA attention, D = 128: query s of sequence b
 *     attends to cache rows 0 .. pos[b] + s (inclusive; positions must stay
 *     below max_ctx) -> out [B * S, Hq, D].  fp32 softmax, P rounded to the
 *     activation type for the P V product. */
int ng_rope_prefill(const void* qkv, void* q_out, void* k_cache, void* v_cache, const int* pos,
                    int dtype, int B, int S, int Hq, int Hkv, int D, float theta, int max_ctx,
                    void* stream);
int ng_attn_prefill(const void* q, const void* k_cache, const void* v_cache, const int* pos, void* out,
                    int dtype, int B, int S, int Hq, int Hkv, int D, int max_ctx, float scale,
                    void* stream);
size_t ng_attn_workspace_bytes(int M, int Hq, int splits);
int ng_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int* ctx_len,
                   void* out, int dtype, int M, int Hq, int Hkv, int D, int max_ctx, int splits,
                   float scale, void* workspace, size_t workspace_bytes, void* stream);
/* ng_rope_append + ng_attn_decode in one pass over the cache: q / K / V are
 * read from qkv [M, (Hq + 2 Hkv) * D], the new K / V row is written at pos[m]
 * (if inside the cache) by the chunk that reads it, and the context is
 * min(pos[m] + 1, max_ctx) rows.  out == NULL: only the split partials are
 * written to the workspace (layout [M][Hq][splits][2 + 128] fp32: running
 * max, sum of exponentials, unnormalised output), for ng_gemv_w4a16_attn. */
int ng_attn_decode_rope(const void* qkv, void* k_cache, void* v_cache, const int* pos, void* out,
                        int dtype, int M, int Hq, int Hkv, int D, int max_ctx, int splits,
                        float scale, float theta, void* workspace, size_t workspace_bytes,
                        void* stream);
int ng_silu_mul(const void* gate_up, void* out, int dtype, int M, int I, void* stream);
/* The cluster decode GEMV (algo 1 fp16 / 2 bf16) with the RMSNorm before it
 * folded into its activation staging: h = x + residual_in, the GEMV input is
 * h * rsqrt(mean(h^2) + eps) * norm_weight (rounded to the activation type, as
 * ng_rmsnorm would store it), and h is written to residual_out (may be NULL;
 * must not alias residual_in -- use two residual buffers alternately).
 * M <= 16; [M, K] activations and residuals, norm_weight [K].  Saves the
 * separate ng_rmsnorm launch before a projection. */
int ng_gemv_w4a16_rmsnorm(const void* x, const void* residual_in, void* residual_out,
                          const void* norm_weight, float eps, int x_dtype, const int32_t* qweight,
                          const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                          void* stream);
/* The same cluster GEMV with the kernel that produces its input folded into
 * the activation staging (no counterpart in the reference, whose decode step
 * is projections only):
 *   ng_gemv_w4a16_silu: X = silu(gate) * up (rounded to x_dtype, as
 *     ng_silu_mul) from gate_up [M, 2K] = gate | up; the SwiGLU before `down`.
 *   ng_gemv_w4a16_attn: X = the attention output combined from the split
 *     partials of ng_attn_decode_rope(out = NULL) [M][K / 128][splits][130],
 *     in split order, bit-identical to the combine of ng_attn_decode_rope.
 * M <= 16; otherwise the arguments of ng_gemv_w4a16. */
int ng_gemv_w4a16_silu(const void* gate_up, int x_dtype, const int32_t* qweight,
                       const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                       void* stream);
int ng_gemv_w4a16_attn(const float* partials, int splits, int x_dtype, const int32_t* qweight,
                       const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                       void* stream);
/*
 * Row-parallel projection fused with its tensor-parallel all-reduce (no
 * counterpart in the reference, which runs on one GPU; replaces
 * ng_gemv_w4a16 + ng_allreduce_sum after the o and down projections): every
 * rank computes its K shard's partial Y with the cluster GEMV (algo 1 fp16 /
 * 2 bf16), and each CTA exchanges its slice of the fp32 partials with the other
 * ranks over NVLink peer memory inside the same kernel (plain stores, one flag
 * per source, bounded waits) and sums them in rank order, so every rank gets
 * the bit-identical full Y.
 *   peer_buffers[p]: rank p's exchange buffer as mapped in this process (the
 *   own one at index `rank`), ng_gemv_allreduce_buffer_bytes(world, N) bytes,
 *   zero-filled before first use (ng_ipc_alloc / ng_ipc_open); one buffer per
 *   (projection width, stream): calls sharing it must not overlap on the GPU.
 *   stage_mode: 0 = X as given, 2 = X = silu(gate) * up from gate_up [M, 2K]
 *   (as ng_gemv_w4a16_silu).  Every rank must call with the same shapes in the
 *   same order.  M <= 16, world 2..8.  A peer that never arrives gives
 *   NG_ERR_DEVICE_TIMEOUT in ng_device_status after 1 s (Y undefined).
 */
size_t ng_gemv_allreduce_buffer_bytes(int world, int N);
int ng_gemv_w4a16_allreduce(const void* x, int x_dtype, const int32_t* qweight, const uint16_t* scales,
                            void* y, int M, int K, int N, int group_size, int stage_mode,
                            void* const* peer_buffers, int rank, int world, void* stream);
/* Row-wise argmax of logits [M, V] (ties: smallest index): value[m] (fp32) and
 * index[m] + index_offset (int64; the offset places a vocab shard).
 * best_scratch: M x 8 bytes, zero before the first call; each call leaves it
 * at zero.  Calls sharing it must not overlap on the GPU. */
int ng_argmax(const void* logits, int dtype, int M, int V, long long index_offset,
              void* best_scratch, float* value, long long* index, void* stream);

/*
 * Output head of the decode step with the argmax fused into its epilogue (no
 * counterpart in the reference, whose decode step stops at the projections,
 * bench/bench_model.py:57-86): for every token m and vocabulary row v of the
 * dense head weight [V, H] (dtype, row-major), logit = x[m] . weight[v] in
 * fp32; keys[m] = max(keys[m], key(logit, index_offset + v)) where
 *   key(l, i) = ((order-preserving bits of l) << 32 | (2^32 - 1 - i)) with the
 *               sign bit flipped,
 * a signed 64-bit value whose maximum is the largest logit and, among equal
 * logits, the smallest index.  Keys combine across vocabulary shards (tensor-
 * parallel ranks) with a MAX all-reduce of int64.  keys must hold LLONG_MIN
 * before the first call (ng_embed_tokens re-arms them); logits [M, V] may be
 * NULL, else it receives the logits rounded to dtype.  x [M, H]; H % 128 == 0,
 * H <= 16384; M <= 64 (weights are re-read per 8 tokens).
 */
int ng_lm_head_argmax(const void* x, const void* weight, int dtype, int M, int V, int H,
                      long long index_offset, void* logits, long long* keys, void* stream);
/*
 * Token embedding gather (no counterpart in the reference): out[m, :] =
 * table[t, :] with t = tokens[m], or, when keys is not NULL, t = the index
 * encoded in keys[m] by ng_lm_head_argmax (keys[m] is then reset to LLONG_MIN
 * and t is written to tokens_out[m] if tokens_out is not NULL).  zero_out
 * (may be NULL) [M, H] is zero-filled (the residual stream of a new step).
 * A token outside [0, V) gives a zero row and sets the device error word
 * (ng_device_status reports it).  out may be NULL (only the token ids are
 * decoded).  H % 8 == 0.
 */
int ng_embed_tokens(const long long* tokens, long long* keys, long long* tokens_out,
                    const void* table, int dtype, int M, int H, long long V, void* out,
                    void* zero_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NIBBLEGEMM_B200_H */
