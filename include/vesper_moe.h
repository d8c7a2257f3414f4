/*
 * vesper_moe.h -- C ABI of the B200 (sm_100a) Mixture-of-Experts FFN forward.
 *
 * Drop-in boundary for VelvetOptimizer's MoE layer.  The reference seam is the
 * nn.Module call `ffn_out, aux_loss = self.ffn(normed)` with
 * `self.ffn = MoELayer(config)` (python/vesper/model.py:402-403, :419-420); the layer
 * itself is python/vesper/model.py:305-385.  Its one native FFI precedent is
 * `extern "C" velvet_complete_update_cuda` (crates/vesper-optimizer/src/cuda/kernels.cu:75-104,
 * declared in crates/vesper-optimizer/src/cuda/velvet.h:8-26 and bound from Rust in
 * crates/vesper-optimizer/src/cuda/mod.rs:9-29): raw device pointers, no stream, no status.
 * This ABI keeps the raw-pointer style and adds an explicit stream, a status code on every
 * call and a per-handle error string.  Plain C types only: no torch or C++ types cross it.
 *
 * Conventions
 *  - every function returns VMOE_OK (0) or a VMOE_ERR_* code; no C++ exception crosses;
 *  - "device pointer" = memory on the handle's device; `stream` is a cudaStream_t
 *    (NULL = legacy default stream);
 *  - matrices are row-major; Linear weights are [out, in] (y = x W^T + b), stacked over
 *    experts on the leading axis, exactly as the reference's nn.Linear parameters;
 *  - one handle per device; calls on one handle must not overlap (not re-entrant);
 *  - vmoe_forward does not synchronise the host on a single GPU.
 */
#ifndef VESPER_MOE_H
#define VESPER_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VMOE_ABI_VERSION 1

#if defined(__GNUC__)
#define VMOE_API __attribute__((visibility("default")))
#else
#define VMOE_API
#endif

/* status codes */
enum {
  VMOE_OK = 0,
  VMOE_ERR_INVALID_ARG = 1,       /* null pointer, bad size, top_k > experts, ...     */
  VMOE_ERR_UNSUPPORTED_SHAPE = 2, /* valid for the reference but not for this build   */
  VMOE_ERR_CUDA = 3,              /* a CUDA runtime/driver call failed                */
  VMOE_ERR_NCCL = 4,              /* reserved for the expert-parallel exchange        */
  VMOE_ERR_TIMEOUT = 5,           /* a bounded device-side wait gave up               */
  VMOE_ERR_DEVICE_STATUS = 6,     /* a kernel reported an error in the status word    */
  VMOE_ERR_NOT_READY = 7,         /* vmoe_forward before vmoe_set_weights             */
  VMOE_ERR_WORKSPACE = 8          /* workspace too small or misaligned                */
};

/* element type of x, out and the weights; every product accumulates in fp32 */
enum { VMOE_F32 = 0, VMOE_BF16 = 1 };

/* Layer configuration.  Mirrors VesperConfig's MoE knobs (python/vesper/config.py:17-22,
 * 33-36) and MoELayer.__init__ (python/vesper/model.py:308-315). */
typedef struct vmoe_config {
  int64_t hidden;       /* H  = hidden_size                                          */
  int64_t inter;        /* I  = intermediate_size (expert d_ff)                      */
  int32_t num_experts;  /* E  = moe_num_experts, >= 2 (config.py:93)                 */
  int32_t top_k;        /* K  = moe_top_k, 1 <= K <= E (config.py:92)                */
  int32_t lora_rank;    /* r  = flylora_rank; 0 = the layer carries no FlyLoRA terms */
  float lora_scaling;   /* flylora_alpha / flylora_rank (model.py:102)               */
  float era_gamma;      /* ERA gamma (config.py:22)                                  */
  int32_t dtype;        /* VMOE_F32 or VMOE_BF16                                     */
  int64_t capacity;     /* max tokens per expert; 0 = no drop (the reference)        */
} vmoe_config;

/* Expert and router weights, as device pointers in the config's dtype (biases too).
 * Shapes use E = num_experts.  The library copies (and repacks) them inside
 * vmoe_set_weights, so the caller may free or modify its buffers afterwards.
 * FlyLoRA tensors may be NULL when lora_rank == 0; a NULL lora_up pair means the
 * branch is off (the reference's zero-initialised lora_up, model.py:120). */
typedef struct vmoe_weights {
  const void* router_w;         /* [E, H]   router.weight                          */
  const void* router_b;         /* [E]      router.bias                            */
  const void* gate_w;           /* [E, I, H] experts.e.gate_proj.base.weight       */
  const void* gate_b;           /* [E, I]                                          */
  const void* up_w;             /* [E, I, H] experts.e.up_proj.base.weight         */
  const void* up_b;             /* [E, I]                                          */
  const void* down_w;           /* [E, H, I] experts.e.down_proj.weight            */
  const void* down_b;           /* [E, H]                                          */
  const void* gate_lora_down_w; /* [E, r, H] experts.e.gate_proj.lora_down.weight  */
  const void* gate_lora_down_b; /* [E, r]                                          */
  const void* gate_lora_up_w;   /* [E, I, r] experts.e.gate_proj.lora_up.weight    */
  const void* gate_lora_up_b;   /* [E, I]                                          */
  const void* up_lora_down_w;   /* [E, r, H]                                       */
  const void* up_lora_down_b;   /* [E, r]                                          */
  const void* up_lora_up_w;     /* [E, I, r]                                       */
  const void* up_lora_up_b;     /* [E, I]                                          */
} vmoe_weights;

typedef struct vmoe_handle vmoe_handle;

/* Create a handle on CUDA device `device`.  Validates the config like
 * VesperConfig.validate (python/vesper/config.py:89-94).  Replaces the constructor
 * MoELayer.__init__ (python/vesper/model.py:308-315). */
VMOE_API int vmoe_create(const vmoe_config* cfg, int device, vmoe_handle** out);

/* Release the handle and every device buffer it owns. */
VMOE_API int vmoe_destroy(vmoe_handle* h);

/* Copy the weights into library-owned device memory in the kernels' layout, folding
 * any FlyLoRA branch into the base projection (the branch is linear, so
 * W + s*U*D and b + s*(U*bd + bu) reproduce base(x) + s*lora_up(lora_down(x)) of
 * python/vesper/model.py:123-126).  Enqueued on `stream`; returns after the copy is
 * enqueued.  Replaces MoELayer's parameter set (load_state_dict).  A second call (after
 * an optimizer step) overwrites the same library buffers in place: it is ordered after
 * forwards enqueued earlier on `stream`, so call it on the stream the forwards use. */
VMOE_API int vmoe_set_weights(vmoe_handle* h, const vmoe_weights* w, void* stream);

/* Bytes of device workspace vmoe_forward needs for `tokens` tokens (256-byte aligned). */
VMOE_API int vmoe_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes);

/* Allocation-free forward.  This entry point has no counterpart in the reference.  It is
 * for callers that cannot allocate device memory when they run the layer (a serving thread
 * under a fixed memory budget, a real-time loop that must not stall on an allocator, an
 * engine without a caching allocator): it behaves exactly like vmoe_forward but takes its
 * scratch from one static device array of VMOE_NO_ALLOC_WORKSPACE_BYTES that every GPU
 * loading this library reserves until the process exits.  It calls no allocator.
 *  - tokens whose vmoe_workspace_size exceeds that size are rejected with
 *    VMOE_ERR_WORKSPACE (e.g. 64 decode tokens at H 2048, I 8192, E 8, K 2 need
 *    about 54 MiB);
 *  - the first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress) -- make that first call before any stream capture;
 *  - all calls share the array: calls whose GPU work overlaps race and corrupt each
 *    other; serialise them.  Nothing needs clearing between calls. */
#define VMOE_NO_ALLOC_WORKSPACE_BYTES (64ull << 20)
VMOE_API int vmoe_forward_no_alloc(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                   float* router_logits, int32_t* topk_idx, float* topk_w,
                                   int32_t* expert_counts, float* aux_loss, void* stream);

/* Where vmoe_forward keeps its intermediates inside the workspace (byte offsets), so a
 * caller can inspect the dispatch: for token t and slot k, slot_of[t*K + k] is the row of
 * the expert-major permuted buffer that holds x[t] (-1 when capacity dropped it); expert
 * e owns rows [expert_offsets[e], expert_offsets[e+1]) (padded to vmoe_segment_align rows), filled
 * in ascending token order like the reference's nonzero() (python/vesper/model.py:347). */
typedef struct vmoe_ws_layout {
  size_t slot_of;        /* int32 [T*K]                                  */
  size_t expert_offsets; /* int32 [E+1]                                  */
  size_t num_tiles;      /* int32 [1]: 128-row tiles in use              */
  size_t x_perm;         /* [max_rows, H] permuted activations           */
  size_t h;              /* [max_rows, I_pad] ERA(gate) * up             */
  size_t y;              /* [max_rows, H_pad] expert outputs             */
  int64_t max_rows;
  int64_t h_ld;          /* row pitch of h in elements                   */
  int64_t y_ld;          /* row pitch of y in elements                   */
  size_t total;          /* == vmoe_workspace_size                       */
} vmoe_ws_layout;
VMOE_API int vmoe_workspace_layout(const vmoe_handle* h, int64_t tokens, vmoe_ws_layout* out);

/* One MoE layer forward over `tokens` rows of x.  Replaces MoELayer.forward
 * (python/vesper/model.py:317-364):
 *   x             [T, H]  device, config dtype (the reference's [B, S, H], flattened)
 *   out           [T, H]  device, config dtype
 *   router_logits [T, E]  fp32, optional (NULL): the router's logits (model.py:322)
 *   topk_idx      [T, K]  int32, optional: chosen experts, probability-descending,
 *                         exact ties broken by lowest expert index (model.py:326)
 *   topk_w        [T, K]  fp32, optional: renormalised gate weights (model.py:329)
 *   expert_counts [E]     int32, optional: assignments per expert (before capacity)
 *   aux_loss      [1]     fp32 device scalar, optional: Switch load-balancing loss
 *                         E * sum_e f_e P_e (model.py:366-385)
 *   workspace             device, >= vmoe_workspace_size bytes, 256-byte aligned
 * All work is enqueued on `stream`; nothing is allocated. */
VMOE_API int vmoe_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                 float* router_logits, int32_t* topk_idx, float* topk_w,
                 int32_t* expert_counts, float* aux_loss,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- training: forward that keeps its intermediates, and the backward -------------------
 * The reference trains through this layer (python/train.py:95-96,465: loss = CE +
 * moe_aux_loss_weight * aux, backward by autograd under bf16 autocast).  These entries are
 * the autograd of MoELayer.forward (python/vesper/model.py:317-385) for bf16 single-GPU
 * handles:
 *  - vmoe_set_training(h, 1, stream) derives transposed copies of the packed weights the
 *    backward GEMMs read (again after every vmoe_set_weights);
 *  - vmoe_forward_train: vmoe_forward's results (out, optional router_logits [T, E] fp32,
 *    aux) that also keeps in `saved`
 *    (vmoe_train_workspace_size) what the backward reads: routing, slots, logits, the
 *    expert inputs, gate|up pre-activations, hidden and expert outputs;
 *  - vmoe_backward: given dout = dL/dout [T, H] and daux = dL/daux (device fp32 scalar,
 *    NULL = 0; the aux-loss weight, 0.01 in the reference), writes dx = dL/dx [T, H] and
 *    the fp32 parameter gradients
 *    below (overwritten, not accumulated).  gate_w / up_w / gate_b / up_b are the gradients
 *    of the effective FlyLoRA weights W + s*U*D and b + s*(U*b_D + b_U) (model.py:123-126),
 *    which are also the base weights' gradients; the LoRA factors' gradients follow as
 *    dU = s*(dW D^T + db b_D^T), db_U = s*db, dD = s*U^T dW, db_D = s*U^T db.
 *  `saved` must be untouched between the two calls; `scratch` is free after the backward. */
typedef struct vmoe_grads {
  float* router_w; /* [E, H]    router.weight            */
  float* router_b; /* [E]                                */
  float* gate_w;   /* [E, I, H] experts.e.gate_proj.base  */
  float* gate_b;   /* [E, I]                             */
  float* up_w;     /* [E, I, H] experts.e.up_proj.base    */
  float* up_b;     /* [E, I]                             */
  float* down_w;   /* [E, H, I] experts.e.down_proj       */
  float* down_b;   /* [E, H]                             */
} vmoe_grads;
VMOE_API int vmoe_set_training(vmoe_handle* h, int enable, void* stream);
VMOE_API int vmoe_train_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* saved_bytes,
                                       size_t* scratch_bytes);
VMOE_API int vmoe_forward_train(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                float* router_logits, float* aux_loss, void* saved,
                                size_t saved_bytes, void* stream);
VMOE_API int vmoe_backward(vmoe_handle* h, const void* x, const void* dout, int64_t tokens,
                           const float* daux, void* dx, const vmoe_grads* grads, const void* saved,
                           size_t saved_bytes, void* scratch, size_t scratch_bytes,
                           void* stream);

/* Fused pre-norm block: the FFN half of TransformerLayer.forward
 * (python/vesper/model.py:418-425) for a MoE layer,
 *     normed = ffn_norm(x);  ffn_out, aux = ffn(normed);  return x + ffn_out, aux
 * in one call.  The LayerNorm is folded into the router's and the dispatch's reads of x
 * (the normalised rows are never written to HBM) and the residual add into the combine.
 * vmoe_set_norm takes the nn.LayerNorm parameters (device, config dtype, [H]; NULL weight =
 * ones, NULL bias = zeros) and its eps (model.py:398-399, config.layer_norm_eps); call it
 * again when they change.  vmoe_forward_residual has vmoe_forward's arguments with
 * x = the residual stream (hidden_states) and out = x + ffn_out (out may equal x); the
 * optional outputs describe the routing of LayerNorm(x).  Workspace: vmoe_workspace_size. */
VMOE_API int vmoe_set_norm(vmoe_handle* h, const void* ln_weight, const void* ln_bias, float eps,
                           void* stream);
VMOE_API int vmoe_forward_residual(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                   float* router_logits, int32_t* topk_idx, float* topk_w,
                                   int32_t* expert_counts, float* aux_loss,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* The same forward with x and out in HOST memory -- the reference's CPU-tensor call of
 * MoELayer.forward (python/vesper/model.py:317-364) served by the GPU.  The batch is cut
 * into `chunks` token chunks (0 = automatic: chunks of >= 8192 tokens, at most 8; at
 * most 16) whose host->device copy, forward and device->host copy overlap on two internal
 * copy streams; outputs are bit-identical to vmoe_forward on the same tokens and aux_loss
 * (host fp32 scalar, optional) is the loss of the whole batch.  Each chunk computes only
 * whole GEMM tiles of its expert segments and carries the remainder rows into the next
 * chunk (the last two chunks pad instead), so the chunks do not each pay the tile padding.
 * With a token capacity (vmoe_config.capacity > 0) the batch is one chunk: the capacity
 * applies to the batch as a whole.
 *   x_host, out_host   [T, H] config dtype; pinned (page-locked) memory for the copies to
 *                      overlap -- pageable memory works but serialises them
 *   workspace          device, >= vmoe_forward_host_workspace_size bytes, 256-byte aligned
 * Enqueued on `stream` (which ends after the last copy): out_host and *aux_loss_host are
 * valid once `stream` has been synchronised. */
VMOE_API int vmoe_forward_host_workspace_size(const vmoe_handle* h, int64_t tokens, int chunks,
                                              size_t* bytes);
VMOE_API int vmoe_forward_host(vmoe_handle* h, const void* x_host, int64_t tokens,
                               void* out_host, float* aux_loss_host, int chunks,
                               void* workspace, size_t workspace_bytes, void* stream);

/* ---- Expert parallelism -------------------------------------------------------------
 * The reference has no distributed code (no collective anywhere in the project); the
 * path's specification partitions this layer expert-parallel: with G ranks, rank r holds
 * experts [r*E/G, (r+1)*E/G) and routes its own tokens.  One forward is three calls with
 * the caller's row exchange (e.g. NCCL all-to-all-v over NVLink) between them:
 *   1. vmoe_ep_route: router over all E experts; each routed (token, k) row of x is
 *      written to send_rows [T*K, H] in expert-major order, unpadded -- so the rows for
 *      destination rank d are contiguous -- and expert_counts[E] (device) says how many;
 *   2. the caller exchanges counts and rows: rank r gathers, for each of its local experts
 *      e, the rows from every source rank into one segment of recv_rows, segments padded
 *      to 128-row tiles; tile_expert[t] = local expert of tile t, *num_tiles = tiles used;
 *   3. vmoe_ep_experts: the local experts' gate|up GEMM with ERA * up and the down GEMM,
 *      recv_rows -> out_rows (same layout);
 *   4. the caller returns each row to its source rank, into back_rows at the position it
 *      had in send_rows;
 *   5. vmoe_ep_combine: out[t] = sum over the token's K rows, ascending expert id, of
 *      w * row, in fp32 -- the same order and arithmetic as vmoe_forward, so each token's
 *      output is bit-identical to the single-GPU forward.
 * Workspaces: vmoe_ep_route and vmoe_ep_combine share one workspace of
 * vmoe_ep_workspace_size(h, tokens, 0) bytes (it carries the routing between them);
 * vmoe_ep_experts takes a different one of vmoe_ep_workspace_size(h, 0, recv_rows_cap)
 * bytes (the received row count is known only after routing).  The aux loss is that of
 * this rank's tokens.  bf16 needs H % 256 == 0; capacity must be 0. */
VMOE_API int vmoe_create_ep(const vmoe_config* cfg, int device, int ep_size, int ep_rank,
                            vmoe_handle** out);
VMOE_API int vmoe_ep_workspace_size(const vmoe_handle* h, int64_t tokens, int64_t recv_rows_cap,
                                    size_t* bytes);
VMOE_API int vmoe_ep_route(vmoe_handle* h, const void* x, int64_t tokens, void* send_rows,
                           int32_t* expert_counts, float* router_logits, float* aux_loss,
                           void* workspace, size_t workspace_bytes, void* stream);
VMOE_API int vmoe_ep_experts(vmoe_handle* h, const void* recv_rows, int64_t recv_rows_cap,
                             const int32_t* tile_expert, const int32_t* num_tiles,
                             void* out_rows, void* workspace, size_t workspace_bytes,
                             void* stream);
VMOE_API int vmoe_ep_combine(vmoe_handle* h, const void* back_rows, int64_t tokens, void* out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Expert parallelism with the exchange fused into the kernels over NVLink peer memory
 * (no collective library, no host synchronisation inside the forward).  Every rank owns
 * one symmetric device region (flags, all ranks' routing counts, a receive buffer and an
 * expert-output buffer) that every peer maps through CUDA IPC:
 *   vmoe_ep_p2p_setup   allocates this rank's regions for up to max_tokens tokens per
 *                       rank per forward, split into `chunks` (1..4) token chunks that run
 *                       on internal streams so one chunk's NVLink exchange overlaps another's
 *                       GEMMs; writes chunks x 64 bytes of CUDA IPC handles to ipc_handles;
 *   (caller)            all-gathers every rank's handles (plain bytes, any transport);
 *   vmoe_ep_p2p_connect maps every peer's regions (G x chunks x 64 bytes, rank-major);
 *   vmoe_ep_p2p_forward one forward: route; publish counts to every peer; dispatch rows
 *                       straight into the owners' receive buffers; local grouped GEMMs;
 *                       combine reading the owners' outputs; device-side epoch flags with
 *                       bounded waits order the ranks.  Same outputs as vmoe_forward.
 * Every rank must call vmoe_ep_p2p_forward the same number of times, each with
 * tokens <= max_tokens.  A bounded wait that gives up (a peer that never arrives) shows up
 * in vmoe_device_status as VMOE_ERR_TIMEOUT. */
VMOE_API int vmoe_ep_p2p_setup(vmoe_handle* h, int64_t max_tokens, int chunks,
                               void* ipc_handles);
VMOE_API int vmoe_ep_p2p_connect(vmoe_handle* h, const void* ipc_handles);
VMOE_API int vmoe_ep_p2p_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes);
VMOE_API int vmoe_ep_p2p_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                 float* router_logits, float* aux_loss, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* vmoe_ep_p2p_forward with x and out in HOST memory (the reference's CPU-tensor call of
 * MoELayer.forward, python/vesper/model.py:317-364, served by this rank's GPU): each token
 * chunk's rows are copied in on an internal copy stream before the chunk starts and copied
 * out as soon as it ends, so the copies overlap the other chunks' exchange and GEMMs (give
 * the handle 2 or more chunks at setup for any overlap).  Outputs are bit-identical to
 * vmoe_ep_p2p_forward; aux_loss_host (optional) is a host fp32 scalar.  x_host / out_host
 * [tokens, H] should be pinned.  Every rank calls it the same number of times, as
 * vmoe_ep_p2p_forward.  Workspace (device, 256-byte aligned):
 * vmoe_ep_p2p_host_workspace_size bytes (routing state plus device staging of max_tokens
 * rows in and out).  Enqueued on `stream`, which ends after the last copy-out. */
VMOE_API int vmoe_ep_p2p_host_workspace_size(const vmoe_handle* h, size_t* bytes);
VMOE_API int vmoe_ep_p2p_forward_host(vmoe_handle* h, const void* x_host, int64_t tokens,
                                      void* out_host, float* aux_loss_host, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ---- Dense FFN -----------------------------------------------------------------------
 * The non-MoE layers' FeedForward (python/vesper/model.py:249-270):
 *   out = down(ERA(gate(x)) * up(x)),  gate/up FlyLoRA linears folded as for the experts,
 * on the same grouped GEMMs as the experts (one expert, no router).  vmoe_ffn_create takes a
 * vmoe_config whose num_experts / top_k / capacity are ignored; vmoe_set_weights then takes
 * the gate/up/down tensors with a leading expert dimension of 1 (router_w may be NULL). */
VMOE_API int vmoe_ffn_create(const vmoe_config* cfg, int device, vmoe_handle** out);
VMOE_API int vmoe_ffn_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes);
VMOE_API int vmoe_ffn_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Read (and clear) the device status word the kernels write when a bounded wait gives
 * up or an index check fails.  Synchronises `stream`.  *code = 0 when all is well. */
VMOE_API int vmoe_device_status(vmoe_handle* h, int32_t* code, void* stream);

/* Per-stage timing, not part of the reference (the benchmark uses it to time the
 * dominant kernel inside its timed region).  vmoe_set_profiling(h, n) makes the next n
 * forwards record CUDA events around each kernel on their stream (n = 0 turns it off);
 * vmoe_stage_times waits for the recorded events, writes the AVERAGE milliseconds per
 * stage over those forwards to ms[0..min(n, stages)-1] (router, scan, plan, dispatch,
 * gemm1_gate_up_era, gemm2_down, combine), the number of forwards averaged to
 * *forwards, and restarts recording. */
VMOE_API int vmoe_set_profiling(vmoe_handle* h, int n);
VMOE_API int vmoe_stage_times(vmoe_handle* h, float* ms, int n, int* n_out, int* forwards);
VMOE_API const char* vmoe_stage_name(int stage);
/* The same for the stages of vmoe_backward (recorded for the next n backwards after
 * vmoe_set_profiling(h, n)). */
VMOE_API int vmoe_backward_stage_times(vmoe_handle* h, float* ms, int n, int* n_out, int* calls);
VMOE_API const char* vmoe_backward_stage_name(int stage);

/* Number of kernel launches the last vmoe_forward enqueued. */
VMOE_API int vmoe_last_launch_count(const vmoe_handle* h);

/* Rows of one grouped-GEMM M tile (128, or 256 when a pair of CTAs shares each tile):
 * expert segments are padded to this, and vmoe_ep_experts' tile_expert has one entry per
 * tile of this many rows.  Not part of the reference. */
VMOE_API int vmoe_gemm_tile_rows(const vmoe_handle* h);

/* Rows each expert segment of the permuted buffer is padded to in a vmoe_forward of
 * `tokens` tokens: vmoe_gemm_tile_rows, or 16 for decode-sized bf16 batches (at most 256
 * tokens), whose GEMMs take the weights as the MMA's M operand and each expert's rows as
 * its N operand.  0 for a null handle or negative tokens.  Not part of the reference. */
VMOE_API int vmoe_segment_align(const vmoe_handle* h, int64_t tokens);

/* Last error message of this handle ("" if none), and a static text per code. */
VMOE_API const char* vmoe_last_error(const vmoe_handle* h);
VMOE_API const char* vmoe_status_string(int status);
VMOE_API int vmoe_abi_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VESPER_MOE_H */
