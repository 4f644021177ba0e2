/*
 * fastb200.h - C ABI of libfastb200.so, the sm_100a (B200) decode hot path of
 * john-jpet/fast-transformer.
 *
 * Conventions shared by every entry point:
 *  - All pointers are DEVICE pointers unless the name says host. Tensors are dense,
 *    row-major, in the layouts documented per function (the reference's layouts).
 *  - `stream` is a cudaStream_t (passed as void* so this header needs no CUDA include).
 *    Every entry point only enqueues work on that stream: no allocation, no host
 *    synchronisation, no device->host read. All of them may be captured in a CUDA graph.
 *  - Return value: FB_OK (0) or a negative status. Arguments are validated on the host
 *    before anything is launched; a failing call launches nothing.
 *  - Device-side waits are bounded. A wait that gives up sets a bit in the library's
 *    device error word and the kernel returns; fb_device_error() reads and clears it.
 *
 * bf16 = IEEE bfloat16 stored as uint16; fp32 = IEEE binary32; int64 = int64_t.
 */
#ifndef FASTB200_H_
#define FASTB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FB_OK 0
#define FB_ERR_ARG (-1)         /* null pointer, negative size, bad enum */
#define FB_ERR_SHAPE (-2)       /* shape outside what the kernels support */
#define FB_ERR_LAUNCH (-3)      /* cudaGetLastError() after the launch */
#define FB_ERR_DRIVER (-4)      /* tensor-map encoder unavailable / refused the map */
#define FB_ERR_WORKSPACE (-5)   /* workspace smaller than the *_workspace() size */
#define FB_ERR_TOO_LARGE (-6)   /* request exceeds a fixed-size entry point's limit */

/* Library version, for the Python loader's sanity check. */
int fb_version(void);

/* Reads the device error word of the current device into *host_flags and clears it.
 * Synchronises the device; call it between steps, never inside a capture. */
int fb_device_error(unsigned int* host_flags);

/* ------------------------------------------------------------------------------------
 * Split-KV GQA decode attention (one query token per row).
 * Replaces engine/kernels/decode_attention.py:238-257 `decode_attention`, whose body
 * `_attend` (:130-149) launches `_decode_partials` (:31-101) then `_decode_merge`
 * (:104-127).
 *
 *   q        bf16 [B, Hq, D]          (the reference's [B, Hq, 1, D])
 *   k, v     bf16 [B, Hkv, C, D]      (one layer's cache, contiguous)
 *   position int64: per_row == 0 -> [1], all rows attend slots [0, position[0]];
 *                   per_row == 1 -> [B], row b attends slots [0, position[b]].
 *            (the reference's scalar form is :246; the per-row form is the
 *             ragged-batch extension of the same rule, valid = position + 1, :48.)
 *   out      bf16 [B, Hq, D]          (the reference's [B, 1, Hq, D])
 *   D in {64, 128}; G = Hq / Hkv in [1, 8].
 *
 * The work is a persistent grid of `ctas` CTAs that split the valid tokens of all
 * (row, KV head) pairs evenly (64-token tiles). fb_decode_attention_ctas() gives the
 * default CTA count (<= 512); fb_decode_attention_workspace() the workspace bytes for a count.
 *
 * fb_decode_attention: the whole operation in one launch; the CTA that finishes a pair last
 *   merges its runs (log-sum-exp combine) in CTA order. The workspace ends with one int
 *   counter per pair: zero it once before its first use; every call leaves it zero again.
 *   Calls that share a workspace must not overlap on the GPU.
 * fb_decode_attention_partials + fb_decode_attention_combine: the same result in two
 *   launches (partials, then the merge kernel), the reference's _decode_partials/_decode_merge
 *   split; no counter state. Both take the same arguments and `ctas`.
 *
 * Launched with programmatic stream serialization: `position`, and the cache slots below it,
 * are read before the wait on the previous kernel, so they must not be written by the kernel
 * launched immediately before on the same stream (in a decode step the position advances at
 * least two kernels earlier); q and the newest slot may come from that kernel.
 * ---------------------------------------------------------------------------------- */
int fb_decode_attention_ctas(int batch, int kv_heads, int capacity, int head_dim);
size_t fb_decode_attention_workspace(int batch, int q_heads, int kv_heads, int head_dim, int ctas);
int fb_decode_attention(const void* q, const void* k, const void* v, const int64_t* position,
                        int per_row, void* out, void* workspace, size_t workspace_bytes, int batch,
                        int q_heads, int kv_heads, int head_dim, int capacity, float scale, int ctas,
                        void* stream);
int fb_decode_attention_partials(const void* q, const void* k, const void* v,
                                 const int64_t* position, int per_row, void* out, void* workspace,
                                 size_t workspace_bytes, int batch, int q_heads, int kv_heads,
                                 int head_dim, int capacity, float scale, int ctas, void* stream);
int fb_decode_attention_combine(const int64_t* position, int per_row, void* out, void* workspace,
                                size_t workspace_bytes, int batch, int q_heads, int kv_heads,
                                int head_dim, int capacity, int ctas, void* stream);
/* Tuning override for fb_decode_attention's cluster form (one shared position, few pairs):
 * every later call uses clusters of `cluster` CTAs (2 to 16) with a `stages`-deep K/V
 * ring (2: three CTAs per SM, 3: two, 4: one); cluster 0 restores the automatic choice.
 * Process-wide; a call whose clusters do not all fit one wave then fails with FB_ERR_SHAPE and
 * launches nothing.
 * For launch-shape sweeps, like the reference's tune.py launch-width search; not needed
 * otherwise. */
int fb_decode_attention_cluster_shape(int cluster, int stages);

/* ------------------------------------------------------------------------------------
 * Decode attention without allocation. No counterpart in the reference.
 * Some callers cannot allocate device memory on the call path: a host runtime that owns a
 * fixed, pre-reserved device pool and hands this library only input and output buffers,
 * or a plugin host whose allocator may not be called from the plugin. They cannot provide
 * fb_decode_attention's workspace, so this entry point uses a fixed scratch array inside
 * the library instead (about 2.7 MiB, held on every GPU that loads the library until the
 * process exits). Same arguments and result as fb_decode_attention, minus the workspace
 * and the CTA count (it uses min(SM count, 160) CTAs). It calls no cudaMalloc/cudaFree.
 *   Limit: batch * kv_heads <= 512 (and the fb_decode_attention limits); a larger request
 *   returns FB_ERR_TOO_LARGE and launches nothing.
 *   The first call on a device looks up the array's device address for that device (it must
 *   be the current device); make that first call before any stream capture. The address is
 *   kept for the life of the process: after cudaDeviceReset (or anything else that destroys
 *   and recreates the device's primary context) this entry point must not be called again.
 *   Every call shares the one array, which keeps the last call's contents; each call clears
 *   the part that must start at zero. Calls that overlap on the GPU (several streams, or
 *   several host threads on one device) race on the array: serialise them.
 * ---------------------------------------------------------------------------------- */
int fb_decode_attention_noalloc(const void* q, const void* k, const void* v,
                                const int64_t* position, int per_row, void* out, int batch,
                                int q_heads, int kv_heads, int head_dim, int capacity, float scale,
                                void* stream);

/* ------------------------------------------------------------------------------------
 * Speculative-verify attention, T > 1 tokens per row, on tcgen05 tensor cores.
 * Replaces engine/kernels/decode_attention.py:637-680 `block_attention` (kernels
 * `_block_partials` :260-350 and `_block_merge` :455-478).
 *   q        bf16 [B, T, Hq, D] token-major; token t of row b sits at slot position[b] + t
 *   k, v     bf16 [B, Hkv, C, D] with the block's own K/V already appended
 *   position int64 [B]; chain int64 [B]: tokens t < chain[b] see slots [0, position[b] + t];
 *            later tokens see [0, position[b]] plus their own slot
 *   out      bf16 [B, T, Hq, D]
 *   D in {64, 128}; T * (Hq / Hkv) <= 2048. `splits` KV splits per (row, KV head):
 *   fb_verify_attention_splits() gives the default; with splits > 1 the workspace must hold
 *   fb_verify_attention_workspace() bytes (partials merged by a second launch).
 * ---------------------------------------------------------------------------------- */
int fb_verify_attention_splits(int batch, int tokens, int kv_heads, int capacity);
size_t fb_verify_attention_workspace(int batch, int tokens, int q_heads, int kv_heads, int splits);
int fb_verify_attention(const void* q, const void* k, const void* v, const int64_t* position,
                        const int64_t* chain, void* out, void* workspace, size_t workspace_bytes,
                        int batch, int tokens, int q_heads, int kv_heads, int head_dim, int capacity,
                        float scale, int splits, void* stream);

/* ------------------------------------------------------------------------------------
 * Fused per-head Q/K RMSNorm + rotate-half RoPE + KV-cache append.
 * Replaces engine/kernels/qk_rope.py:87-129 `qk_rope_cache` (kernel `_qk_rope_cache`
 * :13-84), same cast points: bf16(x * rsqrt(mean(x^2) + eps)) -> bf16(* gain) ->
 * bf16(bf16(w * cos) + bf16(rot(w) * sin)).
 *
 *   packed   bf16 [B*T, (Hq + 2 Hkv) * D] when packed_splits == 0, else fp32 split-K
 *            partials [packed_splits, B*T, (Hq + 2 Hkv) * D] (summed in split order,
 *            then rounded to bf16: engine/kernels/merged.py:37-45)
 *   q_weight, k_weight bf16 [D]
 *   cos, sin bf16: table == 0 -> [rows_of_phase, D] where the phase row of token
 *            (b, t) is t (mode 0/1) or b*T + t (mode 2);
 *            table == 1 -> whole tables [>= C, D] (modes 0 and 2), phase row
 *            p + (phases ? phases[b,t] : t) with p = position[b] (mode 2) or position[0]
 *   position int64: mode 0 (decode)  [1], token t of every row -> slot position[0] + t
 *                   mode 1 (prefill) [T] (unused values), token t -> slot t
 *                   mode 2 (rows)    [B], token t of row b -> slot position[b] + t
 *   phases   int64 [B, T] or NULL (read only when table == 1)
 *   query    bf16 [B, T, Hq, D]       (token-major Q output)
 *   keys, values bf16 [B, Hkv, C, D]  (written in place at the slots above)
 * ---------------------------------------------------------------------------------- */
int fb_qk_norm_rope_append(const void* packed, int packed_splits, const void* q_weight,
                           const void* k_weight, float q_eps, float k_eps, const void* cos,
                           const void* sin, const int64_t* position, const int64_t* phases,
                           void* query, void* keys, void* values, int batch, int tokens,
                           int q_heads, int kv_heads, int head_dim, int capacity, int mode,
                           int table, void* stream);

/* ------------------------------------------------------------------------------------
 * RMSNorm family. Replace engine/kernels/rmsnorm.py:
 *   fb_rmsnorm        <- `rms_norm` :49-72 (kernel :21-46): y = bf16(bf16(x*rsqrt) * w)
 *   fb_add_rmsnorm    <- `add_rms_norm` :98-125 (kernel :75-95):
 *                        sum = bf16(x + residual); out = bf16(bf16(sum*rsqrt) * w)
 *                        x is bf16 [rows, W] (x_splits == 0) or fp32 split partials
 *                        [x_splits, rows, W] (x_splits >= 1).
 *   fb_embed_rmsnorm  <- `embed_rms_norm` :145-162 (kernel :128-142): hidden = table[ids];
 *                        y = rmsnorm(hidden)
 * x/y/residual/out/sum bf16 [rows, W] contiguous (fb_rmsnorm: rows at `row_stride`
 * elements), w bf16 [W]. W <= 16384 and W % 8 == 0.
 * ---------------------------------------------------------------------------------- */
int fb_rmsnorm(const void* x, int64_t row_stride, const void* w, void* y, int rows, int width,
               float eps, void* stream);
int fb_add_rmsnorm(const void* x, int x_splits, const void* residual, const void* w, void* out,
                   void* sum, int rows, int width, float eps, void* stream);
int fb_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, const void* w, void* y,
                     void* hidden, int rows, int width, float eps, void* stream);

/* ------------------------------------------------------------------------------------
 * SwiGLU. Replaces engine/kernels/swiglu.py:27-40 (kernel `_swiglu` :13-24):
 * out = bf16(bf16(g / (1 + exp(-g))) * u) for packed [.., 2I] = [gate | up].
 *   packed bf16 [rows, 2I] (splits == 0) or fp32 partials [splits, rows, 2I] (splits >= 1)
 *   out    bf16 [rows, I]; I % 8 == 0.
 * ---------------------------------------------------------------------------------- */
int fb_swiglu(const void* packed, int splits, void* out, int rows, int width, void* stream);
/* The same on the 64-column blocked layout of fb_linear's SwiGLU weights (block 2i = gate
 * features 64i..64i+63, block 2i+1 = their up features): the split-K companion of epilogue 2
 * (no counterpart in the reference, whose gate/up halves are contiguous). I % 64 == 0. */
int fb_swiglu_blocked(const void* packed, int splits, void* out, int rows, int width, void* stream);

/* ------------------------------------------------------------------------------------
 * Skinny bf16 projection y = x @ W^T with fp32 accumulation and one rounding.
 * Replaces engine/kernels/linear.py:489-523 `linear` for rows <= 64 (the reference's
 * Triton kinds, linear.py:27-93 and gemm.py:51-425; larger row counts stay on cuBLAS
 * exactly as the reference routes them, linear.py:492-493).
 *   x   bf16 [M, K], W bf16 [N, K] (contiguous; K % 8 == 0, N % 8 == 0), M <= 64
 *   epilogue 0: out bf16 [M, N]
 *            1: out fp32 [M, N]
 *            2: SwiGLU: W's rows are [gate; up] interleaved in 64-row blocks (block 2i =
 *               gate rows 64i..64i+63, block 2i+1 = the matching up rows); out bf16 [M, N/2]
 *               = bf16(bf16(silu(bf16(gate))) * bf16(up)) (engine/kernels/swiglu.py:13-24);
 *               N % 128 == 0
 *            3: out fp32 split-K partials [splits, M, N] (split s covers K range
 *               [s*K/splits, (s+1)*K/splits) in 64-wide chunks); consumers sum them in split
 *               order, then round (engine/kernels/merged.py:13-45). No workspace needed.
 * Grid = ceil(N/128) tiles x `splits` K-splits (fb_linear_splits() picks a default for
 * epilogue 3, fb_linear_finished_splits() for epilogues 0-2). For epilogues 0-2 with
 * splits > 1 (at most 8) the CTAs of a tile form a thread-block cluster and sum their
 * partials in split order through distributed shared memory (deterministic; the bits a
 * split consumer produces), in the same launch. No workspace. Launched with programmatic
 * stream serialization (weights are prefetched before the previous kernel completes).
 * ---------------------------------------------------------------------------------- */
int fb_linear_splits(int m, int n, int k);
int fb_linear_finished_splits(int m, int n, int k);
int fb_linear(const void* x, const void* w, void* out, int m, int n, int k, int epilogue, int splits,
              void* stream);

/* ------------------------------------------------------------------------------------
 * Greedy ids without materialized logits: replaces engine/kernels/argmax.py:73-129
 * (`_fused_block_argmax` + `_first_best`, `fused_argmax`) and, in tensor parallelism, the
 * vocabulary-parallel LM head the reference does not have (its argmax is single-GPU).
 * fb_linear_argmax: x bf16 [M, K] (M <= 64) times W bf16 [N, K] (one K split, fp32
 *   accumulation), every logit rounded to bf16 as the projection would store it; each
 *   128-column tile writes its per-row (max, first index) to cand uint64 [M, ceil(N/128)] as
 *   (index_base + column) << 32 | value bits (fb_argmax_candidates_bytes() bytes).
 * fb_argmax_candidates: per row the largest value, ties to the lowest index (torch.argmax's
 *   rule, argmax.py:1-9), into out int64 [rows] (and the winning value into top when not
 *   NULL). With world > 1 each rank holds a vocabulary slice (index_base = its offset) and
 *   the ranks exchange their bests through peer_exchange[r] = rank r's exchange buffer,
 *   uint64 [rows, world, 2], with the flagged-word protocol of fb_reduce_scatter_push (same
 *   epoch rule; bounded 2 s wait): every rank writes the same ids.
 * ---------------------------------------------------------------------------------- */
size_t fb_argmax_candidates_bytes(int m, int n);
int fb_linear_argmax(const void* x, const void* w, int m, int n, int k, int64_t index_base, void* cand,
                     void* stream);
int fb_argmax_candidates(const void* cand, int rows, int tiles, int world, int rank,
                         void* const* peer_exchange, const void* exchange_local, const int64_t* epoch,
                         int64_t* out, float* top, void* stream);

/* ------------------------------------------------------------------------------------
 * Causal GQA prefill attention (flash attention forward, tcgen05): replaces the reference's
 * prefill path engine/attention.py:8-21 (`grouped_sdpa` without a mask: torch SDPA Flash,
 * is_causal, enable_gqa).
 *   q   bf16 [B, Hq, T, D] contiguous (head-major), D = 64 or 128
 *   k,v bf16 [B, Hkv, C, D] (the KV cache; slots [0, T) hold the prompt), C >= T
 *   out bf16 [B, T, Hq, D]: token t of head hq attends keys [0, t] of KV head hq / (Hq/Hkv)
 * fp32 scores and accumulation, P rounded to bf16 for the value product.
 * ---------------------------------------------------------------------------------- */
int fb_prefill_attention(const void* q, const void* k, const void* v, void* out, int batch, int tokens,
                         int q_heads, int kv_heads, int head_dim, int capacity, float scale, void* stream);

/* ------------------------------------------------------------------------------------
 * Speculation bookkeeping (exact speculative decoding): replaces engine/kernels/spec.py's
 * fused programs with the same semantics. All int64 unless noted; one launch each.
 * fb_spec_propose (spec.py:16-124 `_propose`, wrapper `propose` :106-124): per row of
 *   history [B, size], with the newest token at position[b]: tokens [B, T] (trusted token,
 *   chain drafts, alternatives to draft 1), chains [B] = 1 + chain drafts, phases [B, T].
 *   d0..d3 = drafts by match length (<= 1, <= 3, <= 7, longer), each in [1, T - 1];
 *   successor [vocab, top]; stale [B] (a hint, or -1); maxlen = 8 in the reference; T <= 64.
 * fb_spec_within_margin (spec.py:127-166): logits bf16 [B*T, vocab], top fp32 [B*T] (each
 *   row's winning logit): within [B, T] = 1 where draft `slot` >= 1 has a logit within
 *   `margin` of the winning logit of row slot - 1; slot 0 is written 0.
 * fb_spec_settle (spec.py:169-240): accepts, clamps at limit, writes result [B, T + 1]
 *   (gained, then the emitted tokens), history[b, position+1 : position+1+T], move_from
 *   (-1 = no KV move) / move_to, stale, and advances position in place. within may be NULL
 *   (exact acceptance: draft == the model's choice).
 * fb_spec_relocate (spec.py:243-270): store bf16 [planes = 2 x layers, B, Hkv, C, D]: copy
 *   slot move_from[b] to move_to[b] for every head of row b where move_from[b] >= 0.
 * Device-side indices out of range set the error word and skip the access.
 * ---------------------------------------------------------------------------------- */
int fb_spec_propose(const int64_t* history, int64_t size, const int64_t* position, const int64_t* successor,
                    int64_t vocab, int top, const int64_t* stale, int64_t* tokens, int64_t* chains,
                    int64_t* phases, int batch, int tokens_per_row, int d0, int d1, int d2, int d3,
                    int maxlen, void* stream);
int fb_spec_within_margin(const void* logits, int64_t vocab, const int64_t* tokens, const float* top,
                          int64_t* within, int batch, int count, float margin, void* stream);
int fb_spec_settle(const int64_t* tokens, const int64_t* greedy, const int64_t* within, int64_t* position,
                   const int64_t* limit, int64_t* history, int64_t size, int64_t* result,
                   int64_t* move_from, int64_t* move_to, const int64_t* chains, int64_t* stale, int batch,
                   int count, void* stream);
int fb_spec_relocate(void* store, int planes, int batch, int kv_heads, int capacity, int head_dim,
                     const int64_t* move_from, const int64_t* move_to, void* stream);

/* ------------------------------------------------------------------------------------
 * Tensor-parallel all-reduce + residual add + RMSNorm over NVLink peer memory (no counterpart
 * in the reference, which is single-GPU; this replaces an NCCL all-reduce after o_proj/down_proj
 * and the add_rms_norm that follows it, engine/kernels/rmsnorm.py:98-125 arithmetic).
 * Owner-computes: rank q owns columns [q*N/world, (q+1)*N/world) of the N-wide rows.
 * Low-latency protocol: every value travels inside one 8-byte word whose high half is the flag
 * (uint32)(*epoch) + 1, stored whole, so a reader that sees the flag sees the value: no fence,
 * counter or reset. *epoch (a device int64, the decode position) must differ between two calls
 * with the same `use` and stay below 2^31. Each rank owns three uint64 regions (16-byte
 * aligned; zero them before first use and again before *epoch can repeat a value it had):
 *   rs [uses, world, M, N/world]  fp32 partials pushed to this rank as the owner
 *   ag [uses, M, N/2]             summed bf16 pairs of whole rows, from every owner
 *   ss [uses, world, C, M]        each owner's fp32 sums of squares of its slice of a row, per
 *                                 512-column chunk of the slice: C = ceil(N / world / 512) <= 16
 * fb_reduce_scatter_push sums this rank's fp32 split-K partials [splits, M, N] of y = x @ W^T in
 *   split order and stores every value only into the owner's rs[use][rank] (peer_rs[q] =
 *   rank q's rs base). N % (2 * world) == 0.
 * fb_allreduce_add_rmsnorm (one launch): as the owner, polls rs[use] (bounded, 2 s), sums the
 *   ranks in rank order, rounds to bf16, adds `residual` (rounded again: the bf16 residual sum
 *   of add_rms_norm), stores the summed pairs into every rank's ag[use] and the slice's sums of
 *   squares per row and chunk into every rank's ss[use][rank]; then polls its own ag[use] and
 *   ss[use] and writes, for every row, `sum` (the summed row, the next residual) and `out` =
 *   bf16(bf16(sum * rsqrt(mean(sum^2) + eps)) * w), the sums of squares added in rank order and
 *   chunk order (the same bits on every rank). residual/out/sum bf16 [M, N], w bf16 [N]. One call per use per
 *   step, in the same order on every rank.
 * ---------------------------------------------------------------------------------- */
int fb_reduce_scatter_push(const void* partials, int splits, int m, int n, int world, int rank, int use,
                           void* const* peer_rs, const int64_t* epoch, void* stream);
int fb_allreduce_add_rmsnorm(const void* rs, const void* ag, const void* ss, void* const* peer_ag,
                             void* const* peer_ss, int use, int world, int rank, const int64_t* epoch,
                             const void* residual, const void* w, void* out, void* sum, int rows,
                             int width, float eps, void* stream);

/* The same all-reduce + add + RMSNorm in one NVLink phase (push form; no counterpart in the
 * reference, like the owner form above, whose flag protocol and epoch rules it shares). Each
 * rank owns one uint64 region recv [uses, world, M, N] (16-byte aligned, zeroed like the owner
 * form's regions).
 * fb_allreduce_push sums this rank's fp32 split-K partials [splits, M, N] in split order and
 *   stores every value into recv[use][rank] of every rank (peer_recv[q] = rank q's recv base):
 *   world * M * N * 8 bytes per rank and use. N % 2 == 0.
 * fb_allreduce_sum_add_rmsnorm polls its own recv[use] (bounded, 2 s) until every word of every
 *   rank's slab carries the flag, sums the slabs in rank order (the same bits on every rank),
 *   rounds to bf16 and applies add_rms_norm (engine/kernels/rmsnorm.py:75-95 arithmetic):
 *   `sum` = bf16(x + residual), `out` = bf16(bf16(sum * rsqrt(mean(sum^2) + eps)) * w). Each row
 *   is reduced inside one thread-block cluster (no cross-CTA polling), so there is no second
 *   NVLink phase. Measured faster than the owner form at 2 and 4 ranks (config 4).
 * ---------------------------------------------------------------------------------- */
int fb_allreduce_push(const void* partials, int splits, int m, int n, int world, int rank, int use,
                      void* const* peer_recv, const int64_t* epoch, void* stream);
int fb_allreduce_sum_add_rmsnorm(const void* recv, int use, int world, const int64_t* epoch,
                                 const void* residual, const void* w, void* out, void* sum, int rows,
                                 int width, float eps, void* stream);

/* Sums fp32 split partials [splits, count] into bf16 [count] (or fp32 when out_fp32):
 * the reference's `_merge_projection` (linear.py:81-93). */
int fb_merge_splits(const void* partial, int splits, int64_t count, void* out, int out_fp32,
                    void* stream);

/* ------------------------------------------------------------------------------------
 * First-index argmax over bf16 logits. Replaces engine/kernels/argmax.py:51-70 `argmax`
 * (kernels `_block_argmax` :19-33 and `_first_best` :36-48): ties resolve to the lowest
 * index, as torch.argmax.
 *   logits bf16 [rows, vocab]; out int64 [rows]; top fp32 [rows] or NULL (winning logit).
 *   workspace: fb_argmax_workspace(rows, vocab) bytes.
 * ---------------------------------------------------------------------------------- */
size_t fb_argmax_workspace(int rows, int64_t vocab);
int fb_argmax(const void* logits, int rows, int64_t vocab, int64_t* out, float* top,
              void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTB200_H_ */
