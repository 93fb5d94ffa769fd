/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) GatedDeltaNet hot-path library.
 *
 * Every entry point takes plain device pointers, element counts and strides
 * (in ELEMENTS, not bytes) and a cudaStream_t passed as void*.  Nothing here
 * allocates device memory; callers own every buffer, so each call can be
 * captured in a CUDA graph.  Calls are asynchronous on `stream` and return a
 * gdn_status; on failure gdn_last_error() gives a message (thread-local).
 *
 * dtype codes: GDN_F32 = 0, GDN_BF16 = 1.  Unless stated otherwise `dtype`
 * is the type of the activations (q, k, v, x, gate, out, conv state and
 * conv/norm weights); g (log-decay), beta (given as float32, the reference
 * upcasts it before use), recurrent states and A_log / dt_bias are always
 * float32.
 *
 * Slot indexing: pools are [n_slots, ...] arrays; `slot_idx[b]` names the row
 * of the pool that sequence b reads and writes.  A NULL slot_idx means the
 * identity (b -> b).  Slot indices within one call must be distinct and in
 * [0, n_slots); kernels skip out-of-range indices and set *err_flag (when
 * given) to 1 instead of touching memory outside the pool.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * the reference project; "transformers" is models/qwen3_5/modeling_qwen3_5.py
 * of transformers 5.5.x, which the reference patches).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum gdn_status {
  GDN_OK = 0,
  GDN_ERR_ARG = 1,      /* null pointer, negative size, bad enum */
  GDN_ERR_SHAPE = 2,    /* head dims / ratios this library does not build */
  GDN_ERR_DTYPE = 3,    /* dtype code not supported for this entry point */
  GDN_ERR_CUDA = 4,     /* a CUDA launch or attribute call failed */
  GDN_ERR_WORKSPACE = 5 /* workspace missing or too small */
};

enum gdn_dtype { GDN_F32 = 0, GDN_BF16 = 1 };

/* Conv rounding modes (both are the reference's code paths):
 *   GDN_CONV_HF   : fp32 accumulation of the K taps (+bias), one rounding, as
 *                   F.conv1d inside torch_causal_conv1d_update (transformers :210-226)
 *   GDN_CONV_ELEM : products rounded to dtype, fp32 sum rounded, bias added in
 *                   dtype, as elem_conv_update (src/cb_engine.py:43-51)      */
enum gdn_conv_mode { GDN_CONV_HF = 0, GDN_CONV_ELEM = 1 };

/* Message of the last failing call on this thread ("" if none). */
GDN_API const char* gdn_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
GDN_API int gdn_version(void);

/* ---------------------------------------------------------------------------
 * a4. Gated RMSNorm.  Replaces Qwen3_5RMSNormGated.forward (transformers :181-191) and
 * the reference's fused_gated_rmsnorm (src/cb_engine.py:65-67):
 *   y = rnd(w * rnd(x * rsqrt(mean(x^2) + eps))) * silu(float(gate))
 * x, gate, y: [rows, dim] with row strides x_rs, g_rs, y_rs; w: [dim] (dtype).
 * dim <= 1024 and dim % 4 == 0.
 */
GDN_API int gdn_gated_rmsnorm(const void* x, int64_t x_rs, const void* gate, int64_t g_rs,
                      const void* weight, void* y, int64_t y_rs, int64_t rows, int dim,
                      float eps, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * a3. Decode causal depthwise conv with conv-state update.  Replaces
 * elem_conv_update (src/cb_engine.py:43-51) and torch_causal_conv1d_update
 * (transformers :210-226), slot-indexed (src/cb_engine.py:325-328 passes the whole pool).
 *   x: [B, C, T] at x[b*xs_b + c*xs_c + t*xs_t];  y likewise with ys_*.
 *   conv_pool: [n_slots, C, K] contiguous, updated IN PLACE for rows slot_idx[b].
 *   weight: [C, K]; bias: [C] or NULL; activation: 0 none, 1 silu.
 *   K <= 8, T >= 1.
 */
GDN_API int gdn_conv_update(const void* x, int64_t xs_b, int64_t xs_c, int64_t xs_t, void* conv_pool,
                    const int32_t* slot_idx, int64_t n_slots, const void* weight, const void* bias,
                    void* y, int64_t ys_b, int64_t ys_c, int64_t ys_t, int B, int C, int T, int K,
                    int activation, int mode, int dtype, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Prefill causal conv over packed varlen tokens, with conv-state carry and
 * slot scatter.  Replaces the prefill conv of Qwen3_5GatedDeltaNet.forward
 * (transformers :463-474) and of TPEngine.prefill / prefill_chunk (src/cb_tp.py:158-164,
 * :236-244, :260).
 *   x, y: [T_total, C] with token strides xs_t, ys_t (channel stride 1).
 *   cu_seqlens: device int32 [B+1].
 *   conv_pool: [n_slots, C, K]; sequence b starts from conv_pool[slot_idx[b]]
 *   when use_initial != NULL && use_initial[b] != 0 (else zeros), and its
 *   last K inputs are written back to conv_pool[slot_idx[b]].
 *   conv_pool may be NULL (no state read or write).
 */
GDN_API int gdn_prefill_conv(const void* x, int64_t xs_t, void* y, int64_t ys_t, const int32_t* cu_seqlens,
                     int B, void* conv_pool, const int32_t* slot_idx, const int32_t* use_initial,
                     int64_t n_slots, const void* weight, const void* bias, int C, int K,
                     int activation, int dtype, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * a2. Gated delta rule, token by token (decode).  Replaces
 * recurrent_single_step (src/recurrent_single_step.py:8-32) and its T>1
 * fallback torch_recurrent_gated_delta_rule (transformers :314-353).
 *   q, k: [B, T, Hk, dk] at q[b*q_sb + t*q_st + h*dk + i] (likewise k);
 *   v:    [B, T, Hv, dv] at v[b*v_sb + t*v_st + h*dv + i];
 *   g, beta (both f32): [B, T, Hv] at g[b*gb_sb + t*gb_st + h];
 *   out:  [B, T, Hv, dv] at out[b*o_sb + t*o_st + h*dv + i].
 *   v-head h reads q/k head h / (Hv / Hk)  (repeat_interleave semantics).
 *   init_pool [.., Hv, dk, dv] f32 read at init_slot[b] (NULL pool: zeros);
 *   final_pool written at final_slot[b] (NULL pool: not written).  The two
 *   may be the same pool (in-place slot update).
 *   (dk, dv) in {(64,64), (128,128)}; Hv % Hk == 0.
 */
GDN_API int gdn_recurrent(const void* q, int64_t q_sb, int64_t q_st, const void* k, int64_t k_sb,
                  int64_t k_st, const void* v, int64_t v_sb, int64_t v_st, const float* g,
                  const float* beta, int64_t gb_sb, int64_t gb_st, const float* init_pool,
                  const int32_t* init_slot, float* final_pool, const int32_t* final_slot,
                  int64_t n_slots, void* out, int64_t o_sb, int64_t o_st, int B, int T, int Hk,
                  int Hv, int dk, int dv, int use_qk_l2norm, int dtype, int32_t* err_flag,
                  void* stream);

/* ---------------------------------------------------------------------------
 * a5+a3+a2+a4. One fused GDN decode layer for n slots (one token each), the
 * operator part of CBEngine._gdn (src/cb_engine.py:318-352) between the input
 * projections and out_proj:
 *   conv update of mixed_qkv [n, C] (C = 2*Hk*dk + Hv*dv) with the slot's conv
 *   state -> split q|k|v -> beta = sigmoid(b), g = -exp(A_log)*softplus(a+dt_bias)
 *   -> l2norm(q), l2norm(k) -> single-step recurrence on rec_pool[slot_idx]
 *   (in place) -> gated RMSNorm with gate z [n, Hv, dv] -> out [n, Hv, dv].
 *   a, b: [n, Hv] (dtype); A_log, dt_bias: [Hv] f32; norm_w: [dv] (dtype).
 *   z is contiguous and 16-byte aligned (its rows are bulk-copied), as are
 *   rec_pool and the workspace; otherwise GDN_ERR_ARG.
 * dk = dv = 128: two kernels per call, a prep kernel (conv, l2norm, gates)
 * and a persistent state kernel launched as its programmatic dependent; the
 * workspace (gdn_decode_layer_workspace_size() bytes, 16-byte aligned) carries
 * the prepared q/k/v rows [n, C] and gates [n, Hv, 4] f32 between them.
 * dk = dv = 64: one kernel; the workspace holds one uint32 ticket per (slot
 * entry, k-head) that orders the updates of the q/k conv windows shared by a
 * k-head's Hv/Hk value heads.  Zero-fill the workspace before its first use;
 * every call leaves the tickets at zero.
 */
GDN_API size_t gdn_decode_layer_workspace_size(int n, int Hk, int Hv, int dk, int dv, int dtype);

GDN_API int gdn_decode_layer(const void* mixed_qkv, int64_t mixed_rs, const void* z, const void* a,
                     const void* b, const float* A_log, const float* dt_bias, const void* conv_w,
                     const void* conv_b, void* conv_pool, float* rec_pool,
                     const int32_t* slot_idx, int64_t n_slots, const void* norm_w, float eps,
                     void* out, int n, int Hk, int Hv, int dk, int dv, int K, int conv_mode,
                     void* workspace, size_t workspace_bytes, int dtype, int32_t* err_flag,
                     void* stream);

/* gdn_decode_layer with explicit row strides (elements between the rows of
 * consecutive slot entries) for z (z_rs >= Hv*dv), a (a_rs >= Hv) and b
 * (b_rs >= Hv), so that they can be column slices of one fused projection
 * output [n, C + Hv*dv + 2*Hv] (the reference computes them with separate
 * in_proj_z / in_proj_a / in_proj_b GEMMs, src/cb_engine.py:320-323).  z's
 * rows move by 16-byte bulk copies: z and z_rs * element size must be
 * 16-byte aligned.  Everything else as gdn_decode_layer, which is this call
 * with z_rs = Hv*dv and a_rs = b_rs = Hv.
 */
GDN_API int gdn_decode_layer_rows(const void* mixed_qkv, int64_t mixed_rs, const void* z, int64_t z_rs,
                                  const void* a, int64_t a_rs, const void* b, int64_t b_rs,
                                  const float* A_log, const float* dt_bias, const void* conv_w,
                                  const void* conv_b, void* conv_pool, float* rec_pool,
                                  const int32_t* slot_idx, int64_t n_slots, const void* norm_w, float eps,
                                  void* out, int n, int Hk, int Hv, int dk, int dv, int K, int conv_mode,
                                  void* workspace, size_t workspace_bytes, int dtype, int32_t* err_flag,
                                  void* stream);

/* ---------------------------------------------------------------------------
 * gdn_decode_layer for callers that cannot allocate device memory.  This
 * entry point has no counterpart in the reference; the reference never
 * separates workspace from its torch ops.  Hosts such as a serving runtime
 * that owns the whole device-memory budget, or a decode loop that cannot pay
 * cudaMalloc's implicit synchronisation, pass only inputs and outputs here; the
 * workspace is a fixed 8 MiB array inside the library, held by every GPU that
 * loads it until exit.  The array has two parts that never overlap:
 * gdn_decode_layer_noalloc_max_bytes() bytes for the prepared rows and gates
 * of dk = dv = 128 calls (written before they are read), and
 * gdn_decode_layer_noalloc_max_ticket_bytes() bytes for the ticket counters of
 * dk = dv = 64 calls (zero when the library loads; every call that runs to
 * its end leaves them zero, and no dk = 128 call touches them).  Its address
 * is looked up on the first call per device (make that call before any stream
 * capture; do not use the entry point across a cudaDeviceReset).  All calls on
 * a device share that array: calls whose kernels overlap on the GPU race.
 * Requests larger than their part return GDN_ERR_WORKSPACE.  Arguments as
 * gdn_decode_layer minus the workspace.
 */
GDN_API size_t gdn_decode_layer_noalloc_max_bytes(void);
GDN_API size_t gdn_decode_layer_noalloc_max_ticket_bytes(void);

GDN_API int gdn_decode_layer_noalloc(const void* mixed_qkv, int64_t mixed_rs, const void* z, const void* a,
                                     const void* b, const float* A_log, const float* dt_bias,
                                     const void* conv_w, const void* conv_b, void* conv_pool,
                                     float* rec_pool, const int32_t* slot_idx, int64_t n_slots,
                                     const void* norm_w, float eps, void* out, int n, int Hk, int Hv,
                                     int dk, int dv, int K, int conv_mode, int dtype,
                                     int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * a1. Chunked gated delta rule (chunk 64) over packed varlen sequences.
 * Replaces fast_chunk_gated_delta_rule_v2 (src/gdn_chunk_fast2.py:11-62),
 * fast_chunk_gated_delta_rule (src/gdn_chunk_fast.py:65-142) and
 * torch_chunk_gated_delta_rule (transformers :234-311); slot-indexed state read/write
 * replaces the slot copies of src/cb_tp.py:179-180 and :256-261.
 *   q, k: [T_total, Hk, dk] with token strides q_st, k_st; v: [T_total, Hv, dv]
 *   with token stride v_st; g, beta (both f32): [T_total, Hv] token stride
 *   gb_st; out: [T_total, Hv, dv] with token stride o_st.
 *   cu_seqlens: device int32 [B+1].
 *   Sequence b starts from init_pool[init_slot[b]] when init_pool != NULL and
 *   (use_initial == NULL || use_initial[b]); otherwise from zeros.  Its final
 *   state goes to final_pool[final_slot[b]] when final_pool != NULL.
 *   (dk, dv) in {(64,64), (128,128)}; Hv % Hk == 0.
 * GDN_BF16 runs on the tensor cores (bf16 operands, fp32 accumulation and
 * fp32 state); GDN_F32 runs an fp32 CUDA-core path.
 */
GDN_API int gdn_chunk_prefill(const void* q, int64_t q_st, const void* k, int64_t k_st, const void* v,
                      int64_t v_st, const float* g, const float* beta, int64_t gb_st,
                      const int32_t* cu_seqlens, int B, int64_t T_total, const float* init_pool,
                      const int32_t* init_slot, const int32_t* use_initial, float* final_pool,
                      const int32_t* final_slot, int64_t n_slots, void* out, int64_t o_st, int Hk,
                      int Hv, int dk, int dv, int use_qk_l2norm, int dtype, int32_t* err_flag,
                      void* stream);

/* ---------------------------------------------------------------------------
 * a1 with the gate formation of the GDN prefill fused into the kernel.
 * Replaces the gate lines of TPEngine.prefill / prefill_chunk
 * (src/cb_tp.py:170-171, :250-251) and of Qwen3_5GatedDeltaNet.forward
 * (transformers :491-493) together with the
 * chunk rule they feed:
 *   beta = sigmoid(b) rounded to dtype, g = -exp(A_log) * softplus(float(a) + dt_bias)
 * a, b: [T_total, Hv] in dtype with token stride ab_st (the in_proj_a /
 * in_proj_b outputs); A_log, dt_bias: [Hv] f32.  Every other argument is as
 * for gdn_chunk_prefill.  g and beta match the reference's torch expressions
 * bit for bit, so the result equals gdn_chunk_prefill given those tensors.
 */
GDN_API int gdn_chunk_prefill_gates(const void* q, int64_t q_st, const void* k, int64_t k_st, const void* v,
                                    int64_t v_st, const void* a, const void* b, int64_t ab_st,
                                    const float* A_log, const float* dt_bias, const int32_t* cu_seqlens,
                                    int B, int64_t T_total, const float* init_pool, const int32_t* init_slot,
                                    const int32_t* use_initial, float* final_pool, const int32_t* final_slot,
                                    int64_t n_slots, void* out, int64_t o_st, int Hk, int Hv, int dk, int dv,
                                    int use_qk_l2norm, int dtype, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Layer RMSNorm of the hybrid model, Qwen3_5RMSNorm.forward (transformers
 * modeling_qwen3_5.py): y = x * rsqrt(mean(x^2) + eps) * (1 + weight) in fp32,
 * rounded once to dtype; the norm the reference replaces with npu_rms_norm in
 * patch_model (src/cb_engine.py:62-63, 70-71).  x, y: [rows, dim] with row
 * strides x_rs, y_rs (elements); weight [dim] in dtype; dim <= 8192.
 */
GDN_API int gdn_rmsnorm(const void* x, int64_t x_rs, const void* weight, void* y, int64_t y_rs, int64_t rows,
                        int dim, float eps, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Slot-indexed attention decode of the hybrid model's full-attention layers
 * over the engine's KV pool, replacing CBEngine._attn's index_copy_ of the new
 * K/V rows, masked SDPA over a 512-token bucket and sigmoid output gate
 * (src/cb_engine.py:295-316; bucket logic :174-187).  Entry b writes k_new[b],
 * v_new[b] ([kvh, hd]) at position pos[b] of pool row slot_idx[b] (pools
 * [n_slots, kvh, T, hd] bf16) and attends q[b] ([Hq, hd], query head h reads
 * kv head h / (Hq/kvh)) over positions 0..pos[b] with softmax(scale q.k) in
 * fp32; the output [n, Hq, hd] is rounded to bf16 and, when gate is not NULL,
 * multiplied by rnd(sigmoid(gate)) ([n, Hq, hd]) and rounded again.
 * pos[b] < max_len <= T; Hq/kvh <= 8; hd <= 256, a multiple of 8; workspace of
 * gdn_attn_decode_workspace_size(n, Hq, hd, max_len) bytes.  A bad slot or
 * position sets *err_flag = 1 and yields zeros for that entry.
 */
/* The attention layer's decode preamble in one call (CBEngine._attn before the
 * attention, src/cb_engine.py:295-316): from the fused q|gate, k, v projection
 * y [n, 2 Hq hd + 2 kvh hd] (per query head its hd query dims then its hd gate
 * dims; then the kv heads of k, then of v) it writes gdn_attn_decode's inputs
 * q [n, Hq, hd] = rotary(q_norm(q)), k [n, kvh, hd] = rotary(k_norm(k)),
 * v [n, kvh, hd], gate [n, Hq, hd].  q_norm / k_norm: Qwen3_5RMSNorm over hd
 * with gdn_rmsnorm's arithmetic; rotary: apply_rotary_pos_emb on the first rd
 * dims with cos / sin [n, rd] (row stride cs_rs), each bf16 rounding of the
 * torch ops kept -- bit for bit the torch sequence.  bf16; hd a multiple of 8
 * and <= 256; rd a multiple of 16 in 16..hd; 16-byte aligned pointers.
 */
GDN_API int gdn_attn_decode_prep(const void* y, int64_t y_rs, const void* q_norm_w, const void* k_norm_w, float eps,
                                 const void* cos, const void* sin, int64_t cs_rs, int rd, void* q, void* k, void* v,
                                 void* gate, int n, int Hq, int kvh, int hd, int dtype, void* stream);

GDN_API size_t gdn_attn_decode_workspace_size(int n, int Hq, int hd, int max_len);
GDN_API int gdn_attn_decode(const void* q, const void* k_new, const void* v_new, void* kv_k, void* kv_v,
                            int64_t n_slots, int T, const int32_t* slot_idx, const int32_t* pos, int max_len,
                            const void* gate, float scale, void* out, int n, int Hq, int kvh, int hd,
                            void* workspace, size_t workspace_bytes, int dtype, int32_t* err_flag,
                            void* stream);

/* ---------------------------------------------------------------------------
 * a8. Peer-memory all-reduce (sum, bf16) across the ranks of one node, for the
 * row-parallel projections of the TP engine: replaces the NCCL all-reduce of
 * AllReduceLinear.forward (src/cb_tp.py:25-35) for decode-sized outputs.
 * Each rank allocates one buffer of gdn_ar_buffer_bytes(world, max_elems)
 * with gdn_ar_alloc, exports its IPC handle (GDN_IPC_HANDLE_BYTES bytes) with
 * gdn_ar_ipc_handle, opens every other rank's handle with gdn_ar_ipc_open, and
 * passes all world buffer pointers (its own at index rank) to gdn_allreduce.
 * Every rank makes the same sequence of gdn_allreduce calls with the same n
 * (like any collective); x and y may alias; n <= max_elems, n a multiple of 8,
 * x and y 16-byte aligned.  Each rank's result is the fp32 sum of the ranks'
 * inputs in rank order, rounded once to bf16 (identical on every rank).  A
 * rank that does not arrive within spin_limit polls (0: 2^22) makes the
 * others set *err_flag = 3 and leave y untouched; later calls with the same
 * err_flag set stop waiting as soon as they would wait (the ranks are out of
 * step; recreate the buffers).  No multicast memory is
 * used.  Close peer mappings (gdn_ar_ipc_close) and free the buffer
 * (gdn_ar_free) only after every rank's last call has completed.
 */
#define GDN_IPC_HANDLE_BYTES 64
GDN_API size_t gdn_ar_buffer_bytes(int world, size_t max_elems, int dtype);
GDN_API int gdn_ar_alloc(size_t bytes, void** ptr);
GDN_API int gdn_ar_free(void* ptr);
GDN_API int gdn_ar_ipc_handle(void* ptr, void* handle);
GDN_API int gdn_ar_ipc_open(const void* handle, void** ptr);
GDN_API int gdn_ar_ipc_close(void* ptr);
GDN_API int gdn_allreduce(const void* x, void* y, size_t n, int dtype, int rank, int world, void* const* bufs,
                          size_t max_elems, uint32_t spin_limit, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * f1. Decode projections on the tensor cores, and the row-parallel projection
 * fused with its all-reduce.
 *
 * gdn_linear: y[n, n_out] = x[n, k] W[n_out, k]^T (bf16 in, fp32 accumulation,
 * bf16 out), the F.linear of a projection of a decode step
 * (src/cb_engine.py:295-355; nn.Linear without bias), for n = 1..256 tokens.
 * W is streamed once through TMA as the M = 128 operand of tcgen05.mma; the
 * K range of each 128-feature tile is split over the CTAs of a thread-block
 * cluster (splits = 0: chosen from the shape; 1..8: forced) and the partial
 * accumulators are summed through distributed shared memory in split order,
 * so results are deterministic.  No workspace.  Row strides in elements
 * (multiples of 8); x, W, y 16-byte aligned; n_out, k multiples of 8.  A
 * bounded wait that runs out sets *err_flag = 2 (err_flag may be NULL).
 *
 * gdn_linear_allreduce: y = sum over ranks of x_r W_r^T, replacing
 * AllReduceLinear.forward (src/cb_tp.py:25-35: F.linear then dist.all_reduce)
 * in one kernel.  Each rank's product is rounded to bf16 (as the unfused GEMM
 * output) and every 16-feature segment is sent with plain stores to every
 * rank's exchange buffer as soon as its split reduction is done; y is the
 * fp32 sum of the ranks' bf16 partials in rank order, rounded once (identical
 * on every rank).  Buffers: gdn_linear_ar_buffer_bytes(world, max_rows,
 * max_out) bytes per rank from gdn_ar_alloc, shared through gdn_ar_ipc_handle /
 * gdn_ar_ipc_open as for gdn_allreduce; every call on them passes the same
 * max_rows >= n and max_out >= n_out (<= 65536).  Every rank makes the same
 * calls with the same shapes and splits; a rank that does not arrive within
 * spin_limit polls (0: 2^22) makes the others set *err_flag = 3 and leave y
 * unwritten (recreate the buffers).  world = 1 is gdn_linear.  No multicast
 * memory and no bulk/TMA reads of peer memory.
 *
 * With world > 1 every cluster of the launch must be resident at once (a CTA
 * waiting for the other ranks holds its SMs): the split count is lowered until
 * the device holds all tiles' clusters together, else GDN_ERR_SHAPE.
 *
 * gdn_linear_plan fills out[5] (five int32) with the launch gdn_linear (world
 * = 1) or gdn_linear_allreduce (world > 1) makes: splits (CTAs per cluster),
 * pipeline stages, dynamic shared memory bytes per CTA, 128-feature tiles
 * (clusters), 64-wide k-blocks.
 */
GDN_API int gdn_linear(const void* x, int64_t x_rs, const void* w, int64_t w_rs, void* y, int64_t y_rs, int n,
                       int n_out, int k, int splits, int dtype, int32_t* err_flag, void* stream);
GDN_API int gdn_linear_plan(int n, int n_out, int k, int splits, int world, int32_t* out);
GDN_API size_t gdn_linear_ar_buffer_bytes(int world, int max_rows, int max_out, int dtype);
GDN_API int gdn_linear_allreduce(const void* x, int64_t x_rs, const void* w, int64_t w_rs, void* y, int64_t y_rs,
                                 int n, int n_out, int k, int splits, int rank, int world, void* const* bufs,
                                 int max_rows, int max_out, uint32_t spin_limit, int32_t* err_flag, int dtype,
                                 void* stream);

/* f1, split in two for the decode step.  gdn_linear_push is the projection of
 * gdn_linear_allreduce without the wait and the sum: each rank's bf16
 * partial and its flags go to every rank's exchange buffer (so the launch has
 * no residency limit).  gdn_pull_add_rmsnorm then finishes the sum where the
 * decode step continues -- the residual add and the next RMSNorm (the
 * AllReduceLinear output, x + h and Qwen3_5RMSNorm of src/cb_engine.py:
 * 295-355, src/cb_tp.py:25-35) -- in one kernel per token row: it waits
 * (bounded) for every rank's flags of the row's segments, h = bf16(sum of the
 * ranks' partials in rank order), x[j] = bf16(x[j] + h) in place and out[j] =
 * bf16(x[j] * rsqrt(mean(x[j]^2) + eps) * (1 + w)), bit for bit the unfused
 * all-reduce -> add -> gdn_rmsnorm.  Every push must be followed by its pull
 * (same buffers, n_out = dim, rows = n) before the next push.  A rank that does
 * not arrive makes the others set *err_flag = 3 and leave x and out alone.
 * gdn_add_rmsnorm is the same residual add + RMSNorm with h given (one rank).
 * bf16 only; dim a multiple of 8 and <= 8192; rows 16-byte aligned.
 */
GDN_API int gdn_linear_push(const void* x, int64_t x_rs, const void* w, int64_t w_rs, int n, int n_out, int k,
                            int splits, int rank, int world, void* const* bufs, int max_rows, int max_out,
                            int32_t* err_flag, int dtype, void* stream);
/* gdn_allreduce_add_rmsnorm: the all-reduce of a row-parallel projection
 * fused into its consumer, the residual add and the next RMSNorm (the
 * dist.all_reduce of AllReduceLinear.forward, src/cb_tp.py:25-35, then x + h
 * and Qwen3_5RMSNorm, src/cb_engine.py:295-355), one CTA per token row: this
 * rank's partial row h[j] goes to every rank with plain stores and one flag,
 * the other ranks' flags of the row are awaited (bounded), then x[j] =
 * bf16(x[j] + bf16(sum of the partials in rank order)) in place and out[j] =
 * RMSNorm(x[j]) -- bit for bit gdn_allreduce -> add -> gdn_rmsnorm.  Buffers:
 * gdn_ar_norm_buffer_bytes(world, max_rows, dim) per rank from gdn_ar_alloc,
 * shared by IPC like gdn_allreduce's; every call passes the same dim and
 * max_rows >= rows.  A rank that does not arrive makes the others set
 * *err_flag = 3 and leave x and out alone.  bf16; world >= 2.
 */
GDN_API size_t gdn_ar_norm_buffer_bytes(int world, int max_rows, int dim, int dtype);
GDN_API int gdn_allreduce_add_rmsnorm(void* x, int64_t x_rs, const void* h, int64_t h_rs, const void* weight,
                                      void* out, int64_t out_rs, int64_t rows, int dim, float eps, int rank, int world,
                                      void* const* bufs, int max_rows, uint32_t spin_limit, int32_t* err_flag,
                                      int dtype, void* stream);

/* gdn_push_partial: the push of gdn_linear_push for a product y [n, n_out]
 * computed elsewhere (e.g. a library GEMM), same buffers, epochs and flags. */
GDN_API int gdn_push_partial(const void* y, int64_t y_rs, int n, int n_out, int rank, int world, void* const* bufs,
                             int max_rows, int max_out, int dtype, void* stream);
GDN_API int gdn_pull_add_rmsnorm(void* x, int64_t x_rs, const void* weight, void* out, int64_t out_rs, int64_t rows,
                                 int dim, float eps, int rank, int world, void* const* bufs, int max_rows,
                                 int max_out, uint32_t spin_limit, int32_t* err_flag, int dtype, void* stream);
GDN_API int gdn_add_rmsnorm(void* x, int64_t x_rs, const void* h, int64_t h_rs, const void* weight, void* out,
                            int64_t out_rs, int64_t rows, int dim, float eps, int dtype, void* stream);

/* The MLP activation of the decode step, act_fn(gate) * up of Qwen3_5MLP
 * (transformers modeling_qwen3_5.py; the reference runs HF's module,
 * src/cb_engine.py:295-355), on the fused gate|up projection y [rows, 2*inter]
 * (gate = y[:, :inter], up = y[:, inter:]): out = bf16(bf16(silu(gate)) * up),
 * bit for bit the two bf16 torch ops.  bf16; inter a multiple of 8; 16-byte
 * aligned rows.
 */
GDN_API int gdn_silu_mul(const void* y, int64_t y_rs, int inter, void* out, int64_t out_rs, int64_t rows, int dtype,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
