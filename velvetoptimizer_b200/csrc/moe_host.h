// Host-side internals shared by the C-ABI translation units: the handle, the workspace
// plans and the launch helpers of the forward.
//   vesper_moe.cu    handle, weights, the device forward, the dense FeedForward, profiling
//   host_forward.cu  the forward on host buffers (chunked copy-in / compute / copy-out)
//   ep.cu            expert parallelism (NCCL staged and fused NVLink transports)
//   train.cu         the training forward and the backward
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/vesper_moe.h"
#include "kernels.h"

namespace vmoe_host {
using namespace vmoe;

constexpr int kStages = 7;
const char* const kStageNames[kStages] = {"router", "scan", "plan", "dispatch",
                                          "gemm1_gate_up_era", "gemm2_down", "combine"};
constexpr int kBwdStages = 9;
const char* const kBwdStageNames[kBwdStages] = {
    "combine_bwd", "router_bwd", "dh_glu_bwd_gemm", "dx_gemm", "router_dx_gemm", "dx_gather",
    "wgrad_down", "wgrad_gate_up", "wgrad_router"};
// NVTX range names of the stages (host timeline of Nsight Systems; no cost without a tool)
const char* const kNvtxStageNames[kStages] = {
    "vmoe.router", "vmoe.scan", "vmoe.plan", "vmoe.dispatch", "vmoe.gemm1_gate_up_era",
    "vmoe.gemm2_down", "vmoe.combine"};
const char* const kNvtxBwdStageNames[kBwdStages] = {
    "vmoe.bwd.combine", "vmoe.bwd.router", "vmoe.bwd.dh_glu", "vmoe.bwd.dx_gemm",
    "vmoe.bwd.router_dx", "vmoe.bwd.dx_gather", "vmoe.bwd.wgrad_down",
    "vmoe.bwd.wgrad_gate_up", "vmoe.bwd.wgrad_router"};

// One NVTX range per stage: next(i) closes stage i-1's range and opens stage i's (i <
// count); the destructor closes whatever is still open (an error return mid-forward).
struct NvtxStages {
  const char* const* names;
  int count;
  int open = 0;
  NvtxStages(const char* const* n, int c) : names(n), count(c) {}
  void next(int i) {
    if (open) { nvtxRangePop(); open = 0; }
    if (i < count) { nvtxRangePushA(names[i]); open = 1; }
  }
  ~NvtxStages() { if (open) nvtxRangePop(); }
};

constexpr int kGateUpInterleave = 128;  // rows of gate (then up) per 256-row B tile
constexpr int kDownTileN = 256;         // N tile of the down projection

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

constexpr int kMaxChunks = 4;
constexpr int kMaxHostChunks = 16;

// One token chunk's symmetric region and its bookkeeping.
struct P2PChannel {
  char* region = nullptr;
  std::vector<char*> peers;  // every rank's region of this channel as mapped here
  char** peers_dev = nullptr;
  int* block_counter = nullptr;
  unsigned epoch = 0;
};

struct Plan {
  int rb = kTileM;  // tokens per routing block (the router's histograms, the scan, dispatch)
  int nblk = 0;
  int64_t max_tiles = 0, max_rows = 0;
  size_t idx = 0, w = 0, hist = 0, psum = 0, excl = 0, counts = 0, psum_tot = 0, offs = 0,
         tiles = 0, ntiles = 0, aux = 0, slot = 0, stats = 0, xp = 0, h = 0, y = 0, ready = 0,
         total = 0;
};

}  // namespace vmoe_host

using namespace vmoe;
using namespace vmoe_host;

struct vmoe_handle {
  vmoe_config cfg{};
  int device = 0;
  int num_sms = 148;
  int dtype = kF32;
  int64_t H = 0, I = 0, E = 0, K = 0;
  int64_t Ipad = 0, Hpad = 0;
  // expert parallelism: this handle holds experts [ep_rank*E_local, (ep_rank+1)*E_local)
  int ep_size = 1, ep_rank = 0;
  int64_t E_local = 0;
  // expert parallelism over NVLink peer memory (vmoe_ep_p2p_*): one channel per token
  // chunk; every channel has the same region layout
  std::vector<P2PChannel> p2p;
  size_t p2p_sig_off = 0, p2p_counts_off = 0, p2p_recv_off = 0, p2p_y_off = 0;
  // push mode: the down GEMM stores outputs into the source ranks' return buffers
  bool p2p_push = false;
  size_t p2p_ret_off = 0, p2p_back_off = 0;
  int64_t p2p_back_rows = 0;
  int64_t p2p_cap_rows = 0, p2p_max_tokens = 0, p2p_chunk_tokens = 0;
  cudaStream_t p2p_streams[kMaxChunks] = {};
  cudaEvent_t p2p_start = nullptr;
  cudaEvent_t p2p_done[kMaxChunks] = {};
  cudaEvent_t p2p_gemm_done[kMaxChunks] = {};  // orders the chunks' GEMMs one after another
  cudaEvent_t p2p_sent[kMaxChunks] = {};       // and their dispatches
  bool p2p_connected = false;
  int p2p_reserve_sms = 0;  // SMs the chunked GEMMs leave to the transfer kernels
  // host-buffer forward (vmoe_forward_host): copy streams and per-chunk events, made on
  // first use
  cudaStream_t host_in = nullptr, host_out = nullptr;
  cudaEvent_t host_start = nullptr, host_out_done = nullptr;
  cudaEvent_t host_in_ev[kMaxHostChunks] = {}, host_comp_ev[kMaxHostChunks] = {};
  // packed weights (library-owned)
  void* w_r = nullptr;
  float* b_r = nullptr;
  void* w_g = nullptr;  // f32: [E, I, H]; bf16: interleaved gate|up [E, 2*Ipad, H]
  void* w_u = nullptr;  // f32 only
  float* b_g = nullptr; // f32: [E, I]; bf16: interleaved [E, 2*Ipad]
  float* b_u = nullptr;
  void* w_d = nullptr;  // [E, Hpad, Ipad]
  float* b_d = nullptr; // [E, Hpad]
  int* status = nullptr;
  CUtensorMap map_wgu{}, map_wd{};
  // decode-sized forwards (at most decode_max_tokens tokens, bf16): the swapped-operand
  // GEMMs read the packed weights through these maps (64-row gate|up boxes, 128-row down)
  CUtensorMap map_wgu_dec{}, map_wd_dec{};
  int decode_max_tokens = 0;  // 0: never
  bool decode_fused = true;   // both decode GEMMs in one launch (where it pays)
  bool decode_pdl = true;     // decode forwards' kernels with programmatic dependent launch
  bool decode_fold_plan = true;  // decode forwards: scan and plan inside the dispatch
  int l2_bytes = 0;           // the device's L2 size
  // pair GEMM tile order (TcGemmArgs::band_n): -1 = chosen from the weight sizes
  int gemm1_band = -1, gemm2_band = -1;
  int tile_rows = kTileM;  // GEMM M tile: 256 with CTA-pair GEMMs (bf16), else 128
  bool dense = false;      // a dense FeedForward handle (one expert, no router)
  CUtensorMap map_wr{};   // router weights for the tensor-core router (bf16, E <= 64)
  int router_bn = 0;      // its N tile; 0 = CUDA-core router
  // fused pre-norm (vmoe_set_norm / vmoe_forward_residual): LayerNorm weight and bias in
  // fp32, and for the tensor-core router the folded W_r * ln_w, its row sums and the
  // folded bias b_r + W_r ln_b (recomputed whenever the weights or the norm change)
  float* ln_w = nullptr;
  float* ln_b = nullptr;
  float ln_eps = 0.f;
  void* w_r_ln = nullptr;
  float* b_r_ln = nullptr;
  float* c_ln = nullptr;
  CUtensorMap map_wr_ln{};
  bool ln_ready = false;
  // training (vmoe_set_training): transposed copies of the packed weights for the backward
  // GEMMs (every operand K-major): W_d^T [E, Ipad2, Hpad], (gate|up)^T [E, Hpad, 2*Ipad],
  // W_r^T [Hpad, Epad64]
  bool training = false;
  int64_t Ipad2 = 0, Epad64 = 0;
  void* w_dT = nullptr;
  void* w_guT = nullptr;
  void* w_rT = nullptr;
  CUtensorMap map_wdT{}, map_guT{}, map_wrT{};
  bool ready = false;
  // profiling ring: prof_slots forwards x (kStages + 1) events
  int prof_slots = 0;
  int prof_count = 0;
  std::vector<cudaEvent_t> prof_ev;
  // the same for backward stages
  int bprof_count = 0;
  std::vector<cudaEvent_t> bprof_ev;
  int last_launches = 0;
  std::string err;
};

namespace vmoe_host {

// error helpers: record the message on the handle and return the code
int fail(vmoe_handle* h, int code, const char* fmt, ...);
int cuda_fail(vmoe_handle* h, cudaError_t e, const char* what);

// Workspace plan of a single-GPU forward of T tokens routed in blocks of `rb` tokens
// (0: routing_block(h, T)).  The forward must route and dispatch with the plan's rb.
Plan make_plan(const vmoe_handle* h, int64_t T, int rb = 0);

template <typename T>
int alloc(vmoe_handle* h, T** p, size_t bytes, const char* what) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
  if (e != cudaSuccess) return cuda_fail(h, e, what);
  return VMOE_OK;
}

// alloc() unless *p already holds a buffer (whose size the handle's config fixes)
template <typename T>
int alloc_once(vmoe_handle* h, T** p, size_t bytes, const char* what) {
  return *p ? VMOE_OK : alloc(h, p, bytes, what);
}


// Pair GEMM tile order for expert weights (B) of b_bytes per expert: bands of 8 n tiles
// once an expert's B is too large to stay in L2 beside the A tiles and outputs streaming
// through it, row-major otherwise (measured on the gate|up GEMM: 3.55 -> 3.32 ms with 64 MB
// of B per expert, 6.62 -> 7.61 ms with 32 MB, so the switch sits between the two);
// forced >= 0 (VMOE_GEMM1_BAND / VMOE_GEMM2_BAND at handle creation) overrides.
inline int gemm_band(const vmoe_handle* h, int forced, int64_t b_bytes) {
  if (forced >= 0) return forced;
  return b_bytes > static_cast<int64_t>(h->l2_bytes) * 2 / 5 ? 8 : 0;
}

// gate|up GEMM (+ ERA * up) then down GEMM over an expert-major buffer of `max_rows`
// rows (a multiple of 128) whose M tiles map to experts through tiles / ntiles.
template <typename Mark, typename Check>
int run_expert_gemms(vmoe_handle* h, void* xp, int64_t max_rows, const int* tiles,
                     const int* ntiles, void* hb, void* yb, int64_t y_ld, cudaStream_t s,
                     Mark&& mark, Check&& check, int gemm_sms = 0, void* gu_out = nullptr,
                     const P2PArgs* push = nullptr, int64_t a_rows = 0, int64_t out_rows = 0) {
  const int sms = gemm_sms > 0 ? gemm_sms : h->num_sms;  // persistent GEMM grid bound
  const int64_t H = h->H, max_tiles = max_rows / h->tile_rows;
  int rc;
  if (h->dtype == kF32) {
    if ((rc = check(launch_simt_gemm1(static_cast<float*>(xp), H, static_cast<float*>(h->w_g),
                                      static_cast<float*>(h->w_u), h->b_g, h->b_u,
                                      static_cast<float*>(hb), h->Ipad, static_cast<int>(h->I),
                                      static_cast<int>(H), h->cfg.era_gamma, tiles, ntiles,
                                      max_tiles, static_cast<int>(h->E_local), h->status, s),
                    "gemm1")) != VMOE_OK)
      return rc;
    mark();
    return check(launch_simt_gemm2(static_cast<float*>(hb), h->Ipad, static_cast<float*>(h->w_d),
                                   h->b_d, static_cast<float*>(yb), y_ld, static_cast<int>(H),
                                   static_cast<int>(h->Ipad), tiles, ntiles, max_tiles,
                                   static_cast<int>(h->E_local), h->status, s),
                 "gemm2");
  }
  char why[256];
  CUtensorMap map_x, map_h;
  // a_rows < max_rows: A holds only that many rows (the TMA zero-fills the rest of a tile)
  if (!make_tmap_bf16(&map_x, xp, a_rows > 0 ? a_rows : max_rows, H, H, kTileM, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "x_perm tensor map: %s", why);
  if (!make_tmap_bf16(&map_h, hb, max_rows, h->Ipad, h->Ipad, kTileM, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "h tensor map: %s", why);
  TcGemmArgs a1{};
  a1.num_m_tiles = ntiles;
  a1.tile_expert = tiles;
  a1.max_m_tiles = static_cast<int>(max_tiles);
  a1.num_experts = static_cast<int>(h->E_local);
  a1.n_tiles = static_cast<int>(h->Ipad / kGateUpInterleave);
  a1.k_blocks = static_cast<int>((H + 63) / 64);
  a1.b_rows_per_expert = static_cast<int>(2 * h->Ipad);
  a1.out = hb;
  a1.ldo = h->Ipad;
  a1.bias = h->b_g;
  a1.bias_ld = 2 * h->Ipad;
  a1.gamma = h->cfg.era_gamma;
  a1.status = h->status;
  a1.gu_out = gu_out;  // training: keep the pre-activations for the backward
  a1.gu_ld = 2 * h->Ipad;
  const bool pair = h->tile_rows != kTileM;
  a1.band_n = pair ? gemm_band(h, h->gemm1_band, 2 * h->Ipad * H * 2) : 0;
  if ((rc = check(pair ? launch_tc_gemm_pair(true, map_x, h->map_wgu, a1, max_tiles, sms, s)
                       : launch_tc_gemm(true, map_x, h->map_wgu, a1, max_tiles, sms, s),
                  "gemm1")) != VMOE_OK)
    return rc;
  mark();
  TcGemmArgs a2{};
  a2.num_m_tiles = ntiles;
  a2.tile_expert = tiles;
  a2.max_m_tiles = static_cast<int>(max_tiles);
  a2.num_experts = static_cast<int>(h->E_local);
  a2.n_tiles = static_cast<int>(h->Hpad / kDownTileN);
  a2.k_blocks = static_cast<int>(h->Ipad / 64);
  a2.b_rows_per_expert = static_cast<int>(h->Hpad);
  a2.out = yb;
  a2.ldo = y_ld;
  a2.bias = h->b_d;
  a2.bias_ld = h->Hpad;
  a2.gamma = 0.f;
  a2.status = h->status;
  a2.row_limit = out_rows;  // rows past the caller's output are computed but not stored
  a2.band_n = pair ? gemm_band(h, h->gemm2_band, h->Hpad * h->Ipad * 2) : 0;
  if (push) {  // outputs straight into the source ranks' return buffers over NVLink
    a2.push_ret = reinterpret_cast<const int64_t*>(push->peer_base_local + push->ret_off);
    a2.push_peers = push->peer_base;
    a2.push_back_off = push->back_off;
    a2.push_back_rows = push->back_rows;
    a2.push_G = push->G;
    a2.push_epoch = push->epoch;
    a2.ldo = h->H;
    return check(launch_tc_gemm_pair_push(map_h, h->map_wd, a2, max_tiles, sms, s), "gemm2 push");
  }
  return check(pair ? launch_tc_gemm_pair(false, map_h, h->map_wd, a2, max_tiles, sms, s)
                    : launch_tc_gemm(false, map_h, h->map_wd, a2, max_tiles, sms, s),
               "gemm2");
}

// Rows of the packed router weights: E, padded with zero rows to the tensor-core router's
// N tile (bf16, E <= 64) so that its weight boxes stay inside the tensor.
inline int64_t router_rows(const vmoe_handle* h) {
  const int64_t bn = h->dtype == kBF16 ? tc_router_width(static_cast<int>(h->E)) : 0;
  return bn > h->E ? bn : h->E;
}

// Whether a single-GPU forward of T tokens runs the decode-sized (swapped-operand) GEMMs.
inline bool use_decode_gemms(const vmoe_handle* h, int64_t T) {
  return h->dtype == kBF16 && !h->dense && h->ep_size == 1 && T > 0 &&
         T <= h->decode_max_tokens && h->E_local <= kDecodeMaxExperts;
}

// Row alignment of the expert segments in a forward of T tokens.
inline int segment_align(const vmoe_handle* h, int64_t T) {
  return use_decode_gemms(h, T) ? kDecodeRowAlign : h->tile_rows;
}

// Tokens per routing block of a single-GPU forward of T tokens: a decode batch on the
// tensor-core router is routed in blocks of 16 or 32 tokens so that several SMs share its
// x stream (a token's logits are the same in any block); 128 otherwise.
inline int routing_block(const vmoe_handle* h, int64_t T) {
  // from the config alone (tc_router_width, as vmoe_set_weights picks the router), so a
  // workspace sized before the weights are set stays valid
  if (!use_decode_gemms(h, T) || tc_router_width(static_cast<int>(h->E)) == 0) return kTileM;
  return T <= 128 ? 16 : 32;
}

// gate|up GEMM (+ ERA * up) then down GEMM over the expert-major buffer of a decode-sized
// forward: segments padded to kDecodeRowAlign rows at offs[E+1], no tile map.  One
// cooperative launch runs both (`ready`: the per-expert counters the plan kernel zeroed);
// VMOE_DECODE_FUSED=0 at handle creation runs them as two launches instead.
template <typename Mark, typename Check>
int run_decode_gemms(vmoe_handle* h, void* xp, int64_t max_rows, const int* offs, void* hb,
                     void* yb, int64_t T, int* ready, cudaStream_t s, Mark&& mark, Check&& check) {
  const int64_t H = h->H, El = h->E_local;
  char why[256];
  CUtensorMap map_x, map_h;
  if (!make_tmap_bf16(&map_x, xp, max_rows, H, H, kDecodeRowAlign, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "x_perm tensor map: %s", why);
  if (!make_tmap_bf16(&map_h, hb, max_rows, h->Ipad, h->Ipad, kDecodeRowAlign, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "h tensor map: %s", why);
  int64_t n_max = round_up(T, kDecodeRowAlign);
  if (h->cfg.capacity > 0 && round_up(h->cfg.capacity, kDecodeRowAlign) < n_max)
    n_max = round_up(h->cfg.capacity, kDecodeRowAlign);
  DecodeGemmArgs a{};
  a.offs = offs;
  a.num_experts = static_cast<int>(El);
  a.max_rows = max_rows;
  a.n_max = static_cast<int>(n_max);
  a.status = h->status;
  a.bpe1 = static_cast<int>(h->Ipad / 64);
  a.k_blocks1 = static_cast<int>((H + 63) / 64);
  a.a_rows1 = static_cast<int>(2 * h->Ipad);
  a.h = hb;
  a.ldh = h->Ipad;
  a.bias1 = h->b_g;
  a.bias1_ld = 2 * h->Ipad;
  a.gamma = h->cfg.era_gamma;
  a.bpe2 = static_cast<int>(h->Hpad / 128);
  a.k_blocks2 = static_cast<int>(h->Ipad / 64);
  a.a_rows2 = static_cast<int>(h->Hpad);
  a.y = yb;
  a.ldy = h->Hpad;
  a.bias2 = h->b_d;
  a.bias2_ld = h->Hpad;
  // one launch when a down-GEMM work item (128 rows x Ipad) is no larger than a gate|up one
  // (128 rows x H): larger ones, started only once their expert's gate|up blocks are all
  // stored, would end the launch on a few SMs (measured: 166 us in one launch against
  // 153 us in two for 64 tokens at H 2048, I 8192, E 8; 91 against 109 us at I 1024, E 64)
  if (h->decode_fused && a.k_blocks2 <= a.k_blocks1) {
    a.ready = ready;
    const int rc = check(launch_decode_gemm(h->map_wgu_dec, map_x, h->map_wd_dec, map_h, a,
                                            El * (a.bpe1 + a.bpe2), h->num_sms, s),
                         "gemm1 + gemm2 (decode)");
    mark();  // one launch: the gemm2 stage is empty
    return rc;
  }
  DecodeGemmArgs a1 = a, a2 = a;
  a1.bpe2 = 0;
  a2.bpe1 = 0;
  int rc;
  if ((rc = check(launch_decode_gemm(h->map_wgu_dec, map_x, h->map_wd_dec, map_h, a1,
                                     El * a1.bpe1, h->num_sms, s),
                  "gemm1 (decode)")) != VMOE_OK)
    return rc;
  mark();
  return check(launch_decode_gemm(h->map_wgu_dec, map_x, h->map_wd_dec, map_h, a2, El * a2.bpe2,
                                  h->num_sms, s),
               "gemm2 (decode)");
}

// `rb` tokens per routing block (hist / psum rows); below 128 only on the tensor-core router
int run_router(vmoe_handle* h, const void* x, int64_t T, float* logits, int32_t* idx, float* tw,
               int* hist, float* psum, const LnArgs* ln, cudaStream_t s, int rb = kTileM);
int forward_batch(vmoe_handle* h, const void* x, int64_t T, void* out, float* router_logits,
                  int32_t* topk_idx, float* topk_w, int32_t* expert_counts, float* aux_loss,
                  char* ws, const Plan& p, cudaStream_t s, bool prof, float* psum_tot_out,
                  bool prenorm = false);
// The host-buffer forwards' copy streams and per-chunk events, made on first use.
int ensure_host_streams(vmoe_handle* h);
// Transposed copies of the packed weights for the backward GEMMs (training handles).
int make_training_copies(vmoe_handle* h, cudaStream_t s);
// Fold the LayerNorm into the router weights (vmoe_set_norm).
int refold_norm(vmoe_handle* h, cudaStream_t s);

}  // namespace vmoe_host

