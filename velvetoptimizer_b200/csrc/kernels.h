// Internal launcher interface between the C-ABI host code and the CUDA kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vmoe {

enum Dtype { kF32 = 0, kBF16 = 1 };

// ---- programmatic dependent launch ------------------------------------------------------
// While a PdlScope(true) is alive on the launching thread (a decode-sized forward, whose
// kernels each fit in one wave), launches through launch_kernel carry
// cudaLaunchAttributeProgrammaticStreamSerialization: a kernel's launch and the start of its
// CTAs overlap the end of the kernel before it on the stream.  Every kernel launched so waits
// for its predecessor (griddepcontrol.wait) before it touches global memory.
inline thread_local bool g_launch_pdl = false;
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(g_launch_pdl) { g_launch_pdl = on; }
  ~PdlScope() { g_launch_pdl = prev; }
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (g_launch_pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Rows per routing block and per grouped-GEMM M tile: every expert segment of the
// permuted buffer is padded to a multiple of this, so each M tile has one expert.
constexpr int kTileM = 128;

inline size_t dtype_bytes(int dt) { return dt == kF32 ? 4 : 2; }

// ---- fused pre-norm ------------------------------------------------------------------
// LayerNorm over H folded into the router's and the dispatch's read of x (the residual
// stream): per-token (mean, 1/sqrt(var + eps)) in `stats`, affine weight / bias in fp32.
struct LnArgs {
  float2* stats;        // [T]: written by the router (or its statistics pass), read by dispatch
  const float* weight;  // [H]
  const float* bias;    // [H]
  float eps;
};

// ---- routing ------------------------------------------------------------------------
// Router GEMM + softmax + top-K (lowest-index tie-break) + renormalise, per 128-token
// block also the expert histogram hist[blk][E] and probability sums psum[blk][E].  With
// `ln`, the router reads LayerNorm(x) (statistics pass first, rows normalised on load).
cudaError_t launch_router(int dtype, const void* x, const void* w_r, const float* b_r, int64_t T,
                          int H, int E, int K, float* logits, int32_t* topk_idx, float* topk_w,
                          int* hist, float* psum, const LnArgs* ln, cudaStream_t s);

// Per expert: exclusive prefix of hist over blocks (excl[blk][E]), counts, prob sums.
cudaError_t launch_scan_blocks(const int* hist, const float* psum, int nblk, int E, int* excl,
                               int* counts, float* psum_tot, cudaStream_t s);

// Expert offsets padded to `row_align` rows (kTileM for the local GEMMs, 1 for an
// expert-parallel send buffer), M-tile -> expert map (when tile_expert != null), tile
// count, aux loss, caller counts.
cudaError_t launch_plan(const int* counts, const float* psum_tot, int64_t T, int E, int K,
                        int64_t capacity, int row_align, int* offs, int* tile_expert,
                        int* num_tiles, float* aux, int32_t* counts_out, cudaStream_t s,
                        int* zero_e = nullptr);  // [E] ints set to 0 (nullable)

// Token chunks with carried rows (the host-buffer forward): expert e's segment holds the
// carry_in[e] rows carried in from the previous chunk, then this chunk's counts[e] new rows;
// computed[e] of them (whole row_align-row tiles, at least the carried-in rows; everything
// when `last`, i.e. nothing is carried out) are computed now and the rest, at most
// kCarryCap, are carried out.
constexpr int kCarryCap = 256;
cudaError_t launch_plan_carry(const int* counts, const int* carry_in, int E, bool last,
                              int row_align, int* offs, int* computed, int* carry_out,
                              int* tile_expert, int* num_tiles, cudaStream_t s);
// The chunk's dispatch: new rows at positions carry_in[e] + rank of their segment, copied
// when the position is below computed[e], else listed in list_out[e][pos - computed[e]] as
// global (token, k) indices (t0 + t) * K + k with slot -1 for now.  Slots count from
// slot_base.
cudaError_t launch_dispatch_carry(int dtype, const void* x, const int32_t* topk_idx,
                                  const int* excl, const int* offs, int64_t T, int H, int E,
                                  int K, int* slot_of, void* x_perm, int64_t xp_ld,
                                  const int* carry_in, const int* computed, int* list_out,
                                  int64_t t0, int64_t slot_base, int* status, cudaStream_t s);
// The previous chunk's carried-out rows: row x[t] of every listed (t, k) to the first
// carry_in[e] rows of segment e, and its slot (slot_base + row) into the global slot_of.
cudaError_t launch_carry_rows(int dtype, const void* x, int H, int E, int K, const int* list_in,
                              const int* carry_in, const int* offs, void* x_perm, int64_t xp_ld,
                              int64_t slot_base, int* slot_of, int* status, cudaStream_t s);

// Aux loss of a batch routed in chunks: chunk c's per-expert counts (int [E]) and
// probability sums (float [E]) sit at ws + c*stride + counts_off / psum_off.
cudaError_t launch_aux_merge_ws(const void* ws, size_t stride, size_t counts_off, size_t psum_off,
                                int chunks, int64_t T, int E, int K, float* aux, cudaStream_t s);

// Tile map of a dense layer: n tiles, all expert 0.
cudaError_t launch_fill_tiles(int* tile_expert, int n, int* num_tiles, cudaStream_t s);

// The scan and plan of a batch of at most 32 routing blocks, folded into its dispatch:
// every dispatch CTA derives its block's prefixes and the expert offsets (segments padded to
// row_align rows) from the router's histograms, with the same sums as launch_scan_blocks and
// launch_plan; the first CTA writes offs_out [E + 1], the caller's counts, the aux loss and
// zero_n zeros at `zero`.  No tile map is written.
struct DispatchPlan {
  const int* hist;      // [nblk][E]; null: excl and offs come from the scan and plan kernels
  const float* psum;    // [nblk][E]
  int row_align;
  int* offs_out;
  int32_t* counts_out;  // nullable
  float* aux;           // nullable
  int* zero;            // nullable
  int zero_n;
};

// Stable expert-major slots for every (token, k) and the row gather x -> x_perm (with
// `ln`: LayerNorm(x) rows, normalised on the way, rounded to the dtype).  `block_tokens`
// (<= 128) is the routing block the router's histograms and the scan's prefixes use.
cudaError_t launch_dispatch(int dtype, const void* x, const int32_t* topk_idx, const int* excl,
                            const int* offs, int64_t T, int H, int E, int K, int64_t capacity,
                            int* slot_of, void* x_perm, int64_t xp_ld, int* status,
                            const LnArgs* ln, cudaStream_t s, int block_tokens = kTileM,
                            const DispatchPlan* plan = nullptr);

// out[t] = sum over the token's experts in ascending id of w * y[slot]  (fp32 sum); with
// `resid`, out[t] = resid[t] + that sum rounded to the dtype (the residual add of the
// pre-norm block; out may alias resid).
cudaError_t launch_combine(int dtype, const void* y, int64_t y_ld, const int32_t* topk_idx,
                           const float* topk_w, const int* slot_of, int64_t T, int H, int K,
                           void* out, const void* resid, cudaStream_t s);

// ---- fp32 expert GEMMs (CUDA cores; the fp32 correctness path) ------------------------
// h = ERA(A Wg^T + bg) * (A Wu^T + bu) per M tile's expert.
cudaError_t launch_simt_gemm1(const float* a, int64_t lda, const float* wg, const float* wu,
                              const float* bg, const float* bu, float* h, int64_t ldh, int N,
                              int K, float gamma, const int* tile_expert, const int* num_tiles,
                              int64_t max_tiles, int num_experts, int* status, cudaStream_t s);
// y = A Wd^T + bd per M tile's expert.
cudaError_t launch_simt_gemm2(const float* a, int64_t lda, const float* wd, const float* bd,
                              float* y, int64_t ldy, int N, int K, const int* tile_expert,
                              const int* num_tiles, int64_t max_tiles, int num_experts,
                              int* status, cudaStream_t s);

// ---- bf16 expert GEMMs (tcgen05 + TMEM + TMA) ----------------------------------------
struct TcGemmArgs {
  const int* num_m_tiles;   // device scalar, or null: m_tiles_host is used
  int m_tiles_host;
  const int* tile_expert;   // [max_tiles], or null: every tile uses weight block 0
  int max_m_tiles;          // tiles the output buffer holds (bounds num_m_tiles)
  int num_experts;          // experts the weights hold (bounds tile_expert); router: E
  // router epilogue
  int64_t tokens;           // valid rows of A
  int route_rows;           // router: tokens per routing block (M tile), <= 128; 0 = 128
  int top_k;
  float* logits;            // [T, E] or null
  int32_t* topk_idx;        // [T, K]
  float* topk_w;            // [T, K]
  int* hist;                // [ceil(T/128), E]
  float* psum;              // [ceil(T/128), E]
  int n_tiles;              // output tiles per expert along N
  // pair GEMM tile order: 0 = row-major over (m, n); b > 0 = each expert's n tiles in bands
  // of b, every m tile of the expert per band (its band of B stays in L2 across the band)
  int band_n;
  int k_blocks;             // ceil(K / 64)
  int b_rows_per_expert;    // rows of the 2-D weight view per expert
  void* out;                // bf16 output
  int64_t ldo;              // elements
  const float* bias;        // fp32, per expert
  int64_t bias_ld;          // elements per expert
  float gamma;              // ERA gamma (gated epilogue)
  int* status;
  // training: the gated epilogue also stores the pre-activations (gate | up + bias, bf16,
  // same interleaved column layout as the accumulator tile) when gu_out is set
  void* gu_out;
  int64_t gu_ld;
  // GLU backward epilogue (launch_tc_gemm_pair_glu_bwd): reads gu, writes dgu
  const void* gu_in;
  int64_t i_valid;          // columns (of I) that exist: the N tiles may run past Ipad
  // plain epilogue: rows >= row_limit are not stored (0 = no limit), so a GEMM over
  // tile-padded rows can write straight into a caller's [row_limit, N] output
  int64_t row_limit;
  // expert-parallel push epilogue (launch_tc_gemm_pair_push): output row r goes to the
  // source rank's return buffer named by push_ret[r] (see P2PArgs), not to `out`
  const int64_t* push_ret;
  char* const* push_peers;
  size_t push_back_off;
  int64_t push_back_rows;
  int push_G;
  unsigned push_epoch;
  // LayerNorm router (launch_tc_router with ln): b operand = W_r * ln_w, bias = b_r + W_r ln_b
  float2* ln_stats;         // [T] (mean, rstd) out
  const float* ln_c;        // [E] row sums of the folded weights
  float ln_eps;
  int ln_h;                 // H (the normalised width)
};
// gated = true : B tile = [128 gate rows | 128 up rows], h = ERA(gate) * up (128 cols)
// gated = false: plain bias epilogue, 256 output columns per tile
cudaError_t launch_tc_gemm(bool gated, const CUtensorMap& a_map, const CUtensorMap& b_map,
                           const TcGemmArgs& args, int64_t max_tiles, int num_sms,
                           cudaStream_t s);

// Same GEMMs on CTA pairs (tcgen05.mma.cta_group::2): 256-row pair tiles, tile_expert
// holds one expert per 256-row tile, B tensor maps have 128-row boxes (each CTA loads half).
cudaError_t launch_tc_gemm_pair(bool gated, const CUtensorMap& a_map, const CUtensorMap& b_map,
                                const TcGemmArgs& args, int64_t max_pair_tiles, int num_sms,
                                cudaStream_t s);

// Backward of the gated product on CTA pairs: accumulator = dh = dy W_d (the B operand is
// W_d transposed, [E, Ipad2, Hpad]); the epilogue reads the saved pre-activations
// (args.gu_in, interleaved gate|up) and writes dgu = [dh * u * ERA'(g) | dh * ERA(g)] in the
// same interleaved layout (args.out, ldo = 2*Ipad).  No bias.
cudaError_t launch_tc_gemm_pair_glu_bwd(const CUtensorMap& a_map, const CUtensorMap& b_map,
                                        const TcGemmArgs& args, int64_t max_pair_tiles,
                                        int num_sms, cudaStream_t s);

// Plain (bias) epilogue that stores each bf16 output row over NVLink into the source rank's
// return buffer (args.push_*), staged through shared memory so that eight lanes write each
// row's 128 contiguous bytes; rows whose return address carries another epoch (segment
// padding) are skipped.  Every thread fences at system scope before the kernel ends.
cudaError_t launch_tc_gemm_pair_push(const CUtensorMap& a_map, const CUtensorMap& b_map,
                                     const TcGemmArgs& args, int64_t max_pair_tiles, int num_sms,
                                     cudaStream_t s);

// Router on the tensor cores: logits = x W_r^T (+ bias in `args.bias`), softmax, top-K,
// renormalised weights, per-128-token histogram and probability sums.  E <= 64;
// tc_router_width(E) is the N tile (16, 32 or 64), 0 when E is too wide.
// With `ln` the router reads the raw residual stream and applies LayerNorm through the
// folded weights (args.ln_*), writing every token's statistics for the dispatch.
int tc_router_width(int E);
cudaError_t launch_tc_router(const CUtensorMap& x_map, const CUtensorMap& w_map,
                             const TcGemmArgs& args, int num_sms, cudaStream_t s, bool ln);

// ---- decode-sized expert GEMMs (operands swapped: weights are M, the rows are N) --------
// Used when a forward has at most kDecodeMaxTokens tokens: every expert then receives at
// most that many rows, its segment is padded to kDecodeRowAlign rows and becomes the MMA's
// N (16..256); the weights are the M operand, 128 rows per work item.
constexpr int kDecodeMaxTokens = 256;
constexpr int kDecodeRowAlign = 16;
constexpr int kDecodeMaxExperts = 256;
struct DecodeGemmArgs {
  const int* offs;          // [E+1] segment starts (rows), multiples of kDecodeRowAlign
  int num_experts;          // E (<= kDecodeMaxExperts)
  int64_t max_rows;         // rows the activation and output buffers hold
  int n_max;                // largest segment (rows) any expert can have, multiple of 16
                            // (the kernel sizes its ring for the widest one present)
  int* status;
  int64_t row_limit;        // rows >= row_limit are not stored (0 = no limit)
  // phase 1, gate|up (bpe1 = 0: none): h = ERA(gate + bg) * (up + bu)
  int bpe1;                 // work items per expert: 64-feature blocks (Ipad / 64)
  int k_blocks1;            // ceil(H / 64)
  int a_rows1;              // rows of the packed gate|up view per expert (2 * Ipad)
  void* h;                  // bf16 [max_rows, ldh]
  int64_t ldh;
  const float* bias1;       // interleaved gate|up bias [E, bias1_ld]
  int64_t bias1_ld;
  float gamma;              // ERA gamma
  // phase 2, down (bpe2 = 0: none): y = h Wd^T + bd
  int bpe2;                 // work items per expert: 128-feature blocks (Hpad / 128)
  int k_blocks2;            // Ipad / 64
  int a_rows2;              // rows of the packed down view per expert (Hpad)
  void* y;                  // bf16 [max_rows, ldy]
  int64_t ldy;
  const float* bias2;       // [E, bias2_ld], or null
  int64_t bias2_ld;
  // both phases in one launch: [E] counts of each expert's stored gate|up blocks, zero
  // before the launch
  int* ready;
};
// a1_map: packed gate|up weights, 64-row boxes; b1_map: x_perm, 16-row boxes;
// a2_map: packed down weights, 128-row boxes;   b2_map: h, 16-row boxes.
// With bpe1 > 0 and bpe2 > 0 both phases run in one cooperative launch.
cudaError_t launch_decode_gemm(const CUtensorMap& a1_map, const CUtensorMap& b1_map,
                               const CUtensorMap& a2_map, const CUtensorMap& b2_map,
                               const DecodeGemmArgs& args, int64_t max_items, int num_sms,
                               cudaStream_t s);
int decode_gemm_stages(int n_max);

// ---- backward --------------------------------------------------------------------------
// Grouped weight gradient: for e < num_experts, dW_e = A_e^T B_e over the rows of e's
// segment [seg_offs[e], seg_offs[e+1]) (multiples of 64; seg_offs null: one segment of
// seg_rows_host rows), rows_total bounding both.  A [rows, M_total] and B [rows, N_total]
// stay row-major: a_map / b_map are their bf16 tensor maps with 64 x 64 boxes, read
// MN-major by the MMA.  mode 0 writes out[e][m][n] for m < m_valid, n < n_valid; mode 1
// de-interleaves the packed gate|up rows m of 2*Ipad into out (gate) / out2 (up) [e][i][n],
// i < m_valid.  With bias_out, also the column sums of A over the segment (the bias
// gradient) into bias_out (/ bias_out2 in mode 1) [e][i].
struct WgradArgs {
  const int* seg_offs;
  int seg_rows_host;
  int rows_total;
  int num_experts;
  int m_tiles, n_tiles;
  int m_valid, n_valid;
  float* out;
  float* out2;
  int64_t ld_out;
  int64_t out_expert_stride;
  int mode;
  bool vec_ok;              // out / out2 16-byte aligned and ld_out % 4 == 0
  float* bias_out;
  float* bias_out2;
  int* status;
};
cudaError_t launch_wgrad(const CUtensorMap& a_map, const CUtensorMap& b_map, const WgradArgs& args,
                         int num_sms, cudaStream_t s);
// The same on CTA pairs: m_tiles counts 256-row M tiles (M_total padded to 256).
cudaError_t launch_wgrad_pair(const CUtensorMap& a_map, const CUtensorMap& b_map,
                              const WgradArgs& args, int num_sms, cudaStream_t s);

// Batched 2-D transpose of bf16: dst[b][c][r] = src[b][r][c] for r < rows, c < cols, zero in
// the padding of dst ([batch][dst_rows][dst_cols], dst_rows >= cols, dst_cols >= rows).  With
// colsum (fp32 [batch][ceil(rows/64)][cols]) also every 64-row block's column sums.
cudaError_t launch_transpose_bf16(const void* src, int64_t rows, int64_t cols, int64_t src_ld,
                                  int64_t src_batch_stride, int batch, void* dst,
                                  int64_t dst_rows, int64_t dst_cols, int64_t dst_batch_stride,
                                  float* colsum, cudaStream_t s);

// Zero the padding rows [offs[e] + counts[e], offs[e+1]) of every expert segment of buf.
cudaError_t launch_zero_pad_rows(void* buf, int64_t ld_bytes, int64_t row_bytes, const int* offs,
                                 const int* counts, int E, int64_t capacity, cudaStream_t s);

// Combine backward (model.py:337,354-357): for every kept (t, k) with row r = slot_of[t, k],
// dy[r] = bf16(w[t,k] * dout[t]) and dw[t,k] = <dout[t], y[r]> (fp32); dw = 0 for dropped.
cudaError_t launch_combine_bwd(const void* dout, const void* y, int64_t y_ld,
                               const int32_t* topk_idx, const float* topk_w, const int* slot_of,
                               int64_t T, int H, int K, void* dy, int64_t dy_ld, float* dw,
                               cudaStream_t s);

// Router backward (model.py:322-329, 366-385): top-K renormalisation, aux loss and softmax
// gradients from the logits, dw and daux -> dlogits fp32 [T, E] and bf16 [T, e_ld] (zero
// padded to e_ld columns), per-128-token-block column sums [ceil(T/128), E] for the bias.
cudaError_t launch_router_bwd(const float* logits, const int32_t* topk_idx, const float* dw,
                              const int32_t* counts, int64_t T, int E, int K, const float* daux,
                              float* dlogits, void* dl_bf16, int e_ld, float* dl_blocksum,
                              cudaStream_t s);

// dx[t] = sum over the token's kept slots in ascending expert id of dxr[slot] + dxr_router[t]
// (fp32 sum, rounded to bf16).
cudaError_t launch_gather_dx(const void* dxr, int64_t dxr_ld, const void* dxr_router,
                             int64_t router_ld, const int32_t* topk_idx, const int* slot_of,
                             int64_t T, int H, int K, void* dx, cudaStream_t s);

// Sum of fp32 row-block partials per expert: out[e][c] = sum of part[b][c] over the
// 64-row blocks b of e's segment (offs[e] / 64 .. offs[e+1] / 64); with `interleave`, column
// c of the packed gate|up layout goes to out (gate) / out2 (up) at its unpacked index.
cudaError_t launch_segment_sum(const float* part, int64_t part_ld, const int* offs, int E,
                               int cols, int blk_rows, float* out, float* out2, int valid,
                               bool interleave, cudaStream_t s);

// Build a 2-D bf16 tensor map: [rows, cols] row-major with `ld` elements per row, box
// {64 cols, box_rows rows}, 128-byte swizzle.  Returns false on failure.
bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                    uint64_t ld, uint32_t box_rows, char* err, size_t err_len);

// ---- expert parallelism over NVLink peer memory ---------------------------------------
struct P2PArgs {
  char* const* peer_base;   // device array [G]: every rank's symmetric region (own included)
  size_t sig_off, counts_off, recv_off, y_off;
  // push mode (bf16 CTA-pair GEMMs): the down GEMM stores every output row straight into
  // its source rank's return buffer `back` [back_rows, H] (row t*K + k of that rank's chunk);
  // the dispatch writes, for every row it sends, an epoch-tagged return address into the
  // owner's `ret` [cap_rows] int64: epoch << 32 | source rank << 24 | t*K + k
  bool push;
  size_t ret_off, back_off;
  int64_t back_rows;
  char* peer_base_local;    // host-side copy of this rank's own region base (push setup)
  int me, G, E, El, K;
  int64_t H;
  int64_t cap_rows;         // rows of recv / y
  int row_align;            // GEMM tile rows: expert segments are padded to this
  unsigned epoch;           // this forward's flag value
  int* status;
  int* block_counter;       // local, zero between forwards
  int32_t* dest_rank;       // [T*K] owner rank of each (token, k) row
  int32_t* dest_row;        // [T*K] row in the owner's recv / y
  int* tile_expert;         // this rank's GEMM tile map
  int* num_tiles;
};
cudaError_t launch_p2p_publish(const P2PArgs& a, const int* counts, cudaStream_t s);
cudaError_t launch_p2p_wait(const P2PArgs& a, int which, cudaStream_t s);
cudaError_t launch_p2p_signal(const P2PArgs& a, int which, cudaStream_t s);
// spread: the copies of every routing block split over several CTAs (about 2048 in all) --
// for a forward in one token chunk, whose dispatch runs alone; token chunks dispatch while
// other chunks' GEMMs run, and there one CTA per routing block leaves the GEMMs their SMs
cudaError_t launch_p2p_dispatch(int dtype, const P2PArgs& a, const void* x,
                                const int32_t* topk_idx, const int* excl, int64_t T,
                                size_t min_smem, bool spread, cudaStream_t s);
// Push mode: the combine reads every token's K rows from this rank's own return buffer.
cudaError_t launch_p2p_combine_local(int dtype, const P2PArgs& a, const int32_t* topk_idx,
                                     const float* topk_w, int64_t T, void* out, size_t min_smem,
                                     cudaStream_t s);
cudaError_t launch_p2p_combine(int dtype, const P2PArgs& a, const int32_t* topk_idx,
                               const float* topk_w, int64_t T, void* out, size_t min_smem,
                               cudaStream_t s);

// ---- weight packing ------------------------------------------------------------------
// dst[e][map(o)][k] = src[e][o][k] + s * sum_r lu[e][o][r] * ld[e][r][k]  (0 when padded)
struct PackArgs {
  int dtype;                 // of src / lora tensors and dst
  const void* src;           // [E, O, Kin]
  const void* lora_down;     // [E, R, Kin] or null
  const void* lora_up;       // [E, O, R] or null
  int R;
  float scaling;
  int E, O, Kin;
  void* dst;                 // [E, Opad_rows, Kpad] (row map below)
  int Kpad;                  // dst row length
  int dst_rows_per_expert;
  int interleave;            // 0: row o -> o;  >0: block-interleave two matrices (see pack.cu)
  int which;                 // 0 = gate / first, 1 = up / second (interleave only)
};
cudaError_t launch_pack_weight(const PackArgs& a, cudaStream_t s);

// bias: dst[e][map(o)] = b[e][o] + s * (sum_r lu[e][o][r] * bd[e][r] + bu[e][o])  (fp32 out)
struct PackBiasArgs {
  int dtype;
  const void* b;             // [E, O] or null
  const void* lora_up;       // [E, O, R] or null
  const void* lora_down_b;   // [E, R] or null
  const void* lora_up_b;     // [E, O] or null
  int R;
  float scaling;
  int E, O;
  float* dst;
  int dst_per_expert;
  int interleave;
  int which;
};
cudaError_t launch_pack_bias(const PackBiasArgs& a, cudaStream_t s);

// LayerNorm fold into the tensor-core router (bf16 W_r [E, H], fp32 b_r [E], ln_w / ln_b
// fp32 [H]): w_out = bf16(W_r * ln_w), c_out[e] = sum_j w_out[e, j], b_out[e] = b_r[e] +
// sum_j W_r[e, j] ln_b[j] (fixed summation order).
cudaError_t launch_fold_router_ln(const void* w_r, const float* b_r, const float* ln_w,
                                  const float* ln_b, int E, int H, void* w_out, float* b_out,
                                  float* c_out, cudaStream_t s);
// fp32 copy of a [n] vector of the given dtype (null src: fill with `fill`).
cudaError_t launch_to_f32(int dtype, const void* src, int64_t n, float fill, float* dst,
                          cudaStream_t s);

}  // namespace vmoe

// Internal accessors of the opaque handle (defined in vesper_moe.cu).
struct vmoe_handle;
namespace vmoe {
int handle_device(const vmoe_handle* h);
int set_handle_error(vmoe_handle* h, int code, const char* msg);
}  // namespace vmoe
