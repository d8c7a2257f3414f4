// C-ABI host side of the MoE FFN forward (include/vesper_moe.h).
//
// Owns: argument validation (VesperConfig.validate, python/vesper/config.py:89-94), the
// packed weights, the workspace plan, and the launch sequence that replaces
// MoELayer.forward (python/vesper/model.py:317-364):
//
//   router -> scan_blocks -> plan -> dispatch -> gemm1 (gate|up, ERA*up) -> gemm2 (down)
//   -> combine
//
// No host synchronisation and no allocation happen inside vmoe_forward.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <vector>

#include "../../include/vesper_moe.h"
#include "kernels.h"

using namespace vmoe;

namespace {

constexpr int kStages = 7;
const char* const kStageNames[kStages] = {"router", "scan", "plan", "dispatch",
                                          "gemm1_gate_up_era", "gemm2_down", "combine"};
constexpr int kBwdStages = 9;
const char* const kBwdStageNames[kBwdStages] = {
    "combine_bwd", "router_bwd", "dh_glu_bwd_gemm", "dx_gemm", "router_dx_gemm", "dx_gather",
    "wgrad_down", "wgrad_gate_up", "wgrad_router"};
constexpr int kGateUpInterleave = 128;  // rows of gate (then up) per 256-row B tile
constexpr int kDownTileN = 256;         // N tile of the down projection

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

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
  int nblk = 0;
  int64_t max_tiles = 0, max_rows = 0;
  size_t idx = 0, w = 0, hist = 0, psum = 0, excl = 0, counts = 0, psum_tot = 0, offs = 0,
         tiles = 0, ntiles = 0, aux = 0, slot = 0, stats = 0, xp = 0, h = 0, y = 0, total = 0;
};

}  // namespace

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

namespace {

int fail(vmoe_handle* h, int code, const char* fmt, ...) {
  if (h) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    h->err = buf;
  }
  return code;
}

int cuda_fail(vmoe_handle* h, cudaError_t e, const char* what) {
  return fail(h, VMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

Plan make_plan(const vmoe_handle* h, int64_t T) {
  Plan p;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const int64_t E = h->E, K = h->K;
  const size_t elt = dtype_bytes(h->dtype);
  p.nblk = static_cast<int>((T + kTileM - 1) / kTileM);
  const int64_t tr = h->tile_rows;
  int64_t rows_bound = T * K + E * (tr - 1);
  if (h->cfg.capacity > 0) {
    const int64_t cap_rows = E * round_up(h->cfg.capacity, tr);
    if (cap_rows < rows_bound) rows_bound = cap_rows;
  }
  p.max_tiles = (rows_bound + tr - 1) / tr;
  if (p.max_tiles < 1) p.max_tiles = 1;
  p.max_rows = p.max_tiles * tr;
  p.idx = take(T * K * 4);
  p.w = take(T * K * 4);
  p.hist = take(static_cast<size_t>(p.nblk) * E * 4);
  p.psum = take(static_cast<size_t>(p.nblk) * E * 4);
  p.excl = take(static_cast<size_t>(p.nblk) * E * 4);
  p.counts = take(E * 4);
  p.psum_tot = take(E * 4);
  p.offs = take((E + 1) * 4);
  p.tiles = take(p.max_tiles * 4);
  p.ntiles = take(4);
  p.aux = take(4);
  p.slot = take(T * K * 4);
  p.stats = take(T * 8);
  p.xp = take(static_cast<size_t>(p.max_rows) * h->H * elt);
  p.h = take(static_cast<size_t>(p.max_rows) * h->Ipad * elt);
  p.y = take(static_cast<size_t>(p.max_rows) * h->Hpad * elt);
  p.total = off;
  return p;
}

// Workspace of the expert-parallel stages: routing tables (route -> combine) and the
// gate|up activations of up to `recv_rows` received rows.
struct EpPlan {
  int nblk = 0;
  size_t idx = 0, w = 0, hist = 0, psum = 0, excl = 0, counts = 0, psum_tot = 0, offs = 0,
         aux = 0, slot = 0, h = 0, total = 0;
};

EpPlan make_ep_plan(const vmoe_handle* h, int64_t T, int64_t recv_rows) {
  EpPlan p;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const int64_t E = h->E, K = h->K;
  p.nblk = static_cast<int>((T + kTileM - 1) / kTileM);
  p.idx = take(T * K * 4);
  p.w = take(T * K * 4);
  p.hist = take(static_cast<size_t>(p.nblk) * E * 4);
  p.psum = take(static_cast<size_t>(p.nblk) * E * 4);
  p.excl = take(static_cast<size_t>(p.nblk) * E * 4);
  p.counts = take(E * 4);
  p.psum_tot = take(E * 4);
  p.offs = take((E + 1) * 4);
  p.aux = take(4);
  p.slot = take(T * K * 4);
  p.h = take(static_cast<size_t>(recv_rows) * h->Ipad * dtype_bytes(h->dtype));
  p.total = off;
  return p;
}

// Workspace of vmoe_ep_p2p_forward: routing tables, owner rank/row of every routed row,
// this rank's tile map, and the gate|up activations of its receive buffer.
struct P2PPlan {
  int nblk = 0;
  size_t idx = 0, w = 0, hist = 0, psum = 0, excl = 0, counts = 0, psum_tot = 0, offs = 0,
         aux = 0, drank = 0, drow = 0, tiles = 0, ntiles = 0, hbuf = 0, total = 0;
};

P2PPlan make_p2p_plan(const vmoe_handle* h, int64_t T) {
  P2PPlan p;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const int64_t E = h->E, K = h->K, cap = h->p2p_cap_rows;
  p.nblk = static_cast<int>((T + kTileM - 1) / kTileM);
  p.idx = take(T * K * 4);
  p.w = take(T * K * 4);
  p.hist = take(static_cast<size_t>(p.nblk) * E * 4);
  p.psum = take(static_cast<size_t>(p.nblk) * E * 4);
  p.excl = take(static_cast<size_t>(p.nblk) * E * 4);
  p.counts = take(E * 4);
  p.psum_tot = take(E * 4);
  p.offs = take((E + 1) * 4);
  p.aux = take(4);
  p.drank = take(T * K * 4);
  p.drow = take(T * K * 4);
  p.tiles = take((cap / h->tile_rows + 1) * 4);
  p.ntiles = take(4);
  p.hbuf = take(static_cast<size_t>(cap) * h->Ipad * dtype_bytes(h->dtype));
  p.total = off;
  return p;
}

void free_weights(vmoe_handle* h) {
  void* bufs[] = {h->w_r, h->b_r, h->w_g, h->w_u, h->b_g, h->b_u, h->w_d, h->b_d,
                  h->w_r_ln, h->b_r_ln, h->c_ln};
  for (void* b : bufs)
    if (b) cudaFree(b);
  h->w_r = h->w_g = h->w_u = h->w_d = h->w_r_ln = nullptr;
  h->b_r = h->b_g = h->b_u = h->b_d = h->b_r_ln = h->c_ln = nullptr;
  h->ready = false;
  h->ln_ready = false;
}

int validate_config(const vmoe_config* c, char* why, size_t n) {
  if (c->hidden <= 0 || c->inter <= 0) {
    snprintf(why, n, "hidden (%lld) and inter (%lld) must be positive",
             static_cast<long long>(c->hidden), static_cast<long long>(c->inter));
    return VMOE_ERR_INVALID_ARG;
  }
  if (c->num_experts < 2) {  // config.py:94
    snprintf(why, n, "num_experts must be >= 2 (got %d)", c->num_experts);
    return VMOE_ERR_INVALID_ARG;
  }
  if (c->top_k < 1 || c->top_k > c->num_experts) {  // config.py:92
    snprintf(why, n, "top_k must satisfy 1 <= top_k <= num_experts (got top_k=%d, E=%d)",
             c->top_k, c->num_experts);
    return VMOE_ERR_INVALID_ARG;
  }
  if (c->dtype != VMOE_F32 && c->dtype != VMOE_BF16) {
    snprintf(why, n, "dtype must be VMOE_F32 or VMOE_BF16 (got %d)", c->dtype);
    return VMOE_ERR_INVALID_ARG;
  }
  if (c->capacity < 0 || c->lora_rank < 0) {
    snprintf(why, n, "capacity and lora_rank must be >= 0");
    return VMOE_ERR_INVALID_ARG;
  }
  if (c->num_experts > 256) {
    snprintf(why, n, "num_experts > 256 is not supported by this build (got %d)", c->num_experts);
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  if (c->top_k > 32) {
    snprintf(why, n, "top_k > 32 is not supported by this build (got %d)", c->top_k);
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  if (c->hidden % 8 || c->inter % 8) {
    snprintf(why, n, "hidden and inter must be multiples of 8 (got %lld, %lld)",
             static_cast<long long>(c->hidden), static_cast<long long>(c->inter));
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  if (c->lora_rank > 1024) {
    snprintf(why, n, "lora_rank > 1024 is not supported (got %d)", c->lora_rank);
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  return VMOE_OK;
}

template <typename T>
int alloc(vmoe_handle* h, T** p, size_t bytes, const char* what) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
  if (e != cudaSuccess) return cuda_fail(h, e, what);
  return VMOE_OK;
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

// Router + softmax + top-K + per-block histogram / probability sums: on the tensor cores
// for bf16 with E <= 64, on CUDA cores otherwise (fp32 parity, or wider routers).
// With `ln` the router reads LayerNorm(x) without materialising it: the tensor-core router
// through the folded weights (and its own row statistics), the CUDA-core router through a
// statistics pass and normalisation on load.
int run_router(vmoe_handle* h, const void* x, int64_t T, float* logits, int32_t* idx, float* tw,
               int* hist, float* psum, const LnArgs* ln, cudaStream_t s) {
  const int64_t H = h->H;
  cudaError_t e;
  if (h->dtype == kBF16 && h->router_bn > 0) {
    char why[256];
    CUtensorMap map_x;
    if (!make_tmap_bf16(&map_x, x, T, H, H, kTileM, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "x tensor map: %s", why);
    TcGemmArgs a{};
    a.num_m_tiles = nullptr;
    a.m_tiles_host = static_cast<int>((T + kTileM - 1) / kTileM);
    a.tile_expert = nullptr;
    a.max_m_tiles = a.m_tiles_host;
    a.num_experts = static_cast<int>(h->E);
    a.n_tiles = 1;
    a.k_blocks = static_cast<int>((H + 63) / 64);
    a.b_rows_per_expert = 0;
    a.bias = h->b_r;
    a.status = h->status;
    a.tokens = T;
    a.top_k = static_cast<int>(h->K);
    a.logits = logits;
    a.topk_idx = idx;
    a.topk_w = tw;
    a.hist = hist;
    a.psum = psum;
    if (ln) {
      a.bias = h->b_r_ln;
      a.ln_stats = ln->stats;
      a.ln_c = h->c_ln;
      a.ln_eps = ln->eps;
      a.ln_h = static_cast<int>(H);
    }
    e = launch_tc_router(map_x, ln ? h->map_wr_ln : h->map_wr, a, h->num_sms, s, ln != nullptr);
  } else {
    e = launch_router(h->dtype, x, h->w_r, h->b_r, T, static_cast<int>(H), static_cast<int>(h->E),
                      static_cast<int>(h->K), logits, idx, tw, hist, psum, ln, s);
  }
  if (e != cudaSuccess) return cuda_fail(h, e, "router");
  h->last_launches += (ln && !(h->dtype == kBF16 && h->router_bn > 0)) ? 2 : 1;
  return VMOE_OK;
}

// One single-GPU forward of T >= 1 tokens on stream s, workspace laid out by make_plan(h, T).
// psum_tot_out (nullable) takes the batch's per-expert probability sums instead of the
// workspace, so that a chunked caller can merge the aux loss of the whole batch.
// With prenorm, x is the residual stream: the layer runs on LayerNorm(x) (folded into the
// router's and the dispatch's reads) and out = x + MoE(LayerNorm(x)).
int forward_batch(vmoe_handle* h, const void* x, int64_t T, void* out, float* router_logits,
                  int32_t* topk_idx, float* topk_w, int32_t* expert_counts, float* aux_loss,
                  char* ws, const Plan& p, cudaStream_t s, bool prof, float* psum_tot_out,
                  bool prenorm = false) {
  const int64_t E = h->E, K = h->K, H = h->H;
  LnArgs ln_args{reinterpret_cast<float2*>(ws + p.stats), h->ln_w, h->ln_b, h->ln_eps};
  const LnArgs* ln = prenorm ? &ln_args : nullptr;
  int32_t* idx = topk_idx ? topk_idx : reinterpret_cast<int32_t*>(ws + p.idx);
  float* tw = topk_w ? topk_w : reinterpret_cast<float*>(ws + p.w);
  int* hist = reinterpret_cast<int*>(ws + p.hist);
  float* psum = reinterpret_cast<float*>(ws + p.psum);
  int* excl = reinterpret_cast<int*>(ws + p.excl);
  int* counts = reinterpret_cast<int*>(ws + p.counts);
  float* psum_tot = psum_tot_out ? psum_tot_out : reinterpret_cast<float*>(ws + p.psum_tot);
  int* offs = reinterpret_cast<int*>(ws + p.offs);
  int* tiles = reinterpret_cast<int*>(ws + p.tiles);
  int* ntiles = reinterpret_cast<int*>(ws + p.ntiles);
  float* aux = aux_loss ? aux_loss : reinterpret_cast<float*>(ws + p.aux);
  int* slot = reinterpret_cast<int*>(ws + p.slot);
  void* xp = ws + p.xp;
  void* hb = ws + p.h;
  void* yb = ws + p.y;

  cudaEvent_t* ev = prof ? &h->prof_ev[static_cast<size_t>(h->prof_count) * (kStages + 1)] : nullptr;
  int stage = 0;
  auto mark = [&]() {
    if (prof) cudaEventRecord(ev[stage], s);
    ++stage;
  };
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  int rc;
  mark();
  if ((rc = run_router(h, x, T, router_logits, idx, tw, hist, psum, ln, s)) != VMOE_OK) return rc;
  mark();
  if ((rc = check(launch_scan_blocks(hist, psum, p.nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s),
                  "scan")) != VMOE_OK)
    return rc;
  mark();
  if ((rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K),
                              h->cfg.capacity, static_cast<int>(h->tile_rows), offs, tiles,
                              ntiles, aux, expert_counts, s),
                  "plan")) != VMOE_OK)
    return rc;
  mark();
  if ((rc = check(launch_dispatch(h->dtype, x, idx, excl, offs, T, static_cast<int>(H),
                                  static_cast<int>(E), static_cast<int>(K), h->cfg.capacity, slot,
                                  xp, H, h->status, ln, s),
                  "dispatch")) != VMOE_OK)
    return rc;
  mark();
  if ((rc = run_expert_gemms(h, xp, p.max_rows, tiles, ntiles, hb, yb, h->Hpad, s, mark,
                             check)) != VMOE_OK)
    return rc;
  mark();
  if ((rc = check(launch_combine(h->dtype, yb, h->Hpad, idx, tw, slot, T, static_cast<int>(H),
                                 static_cast<int>(K), out, prenorm ? x : nullptr, s),
                  "combine")) != VMOE_OK)
    return rc;
  mark();
  return VMOE_OK;
}

}  // namespace

namespace vmoe {
int handle_device(const vmoe_handle* h) { return h ? h->device : -1; }
int set_handle_error(vmoe_handle* h, int code, const char* msg) { return fail(h, code, "%s", msg); }
}  // namespace vmoe

extern "C" {

int vmoe_abi_version(void) { return VMOE_ABI_VERSION; }

const char* vmoe_status_string(int status) {
  switch (status) {
    case VMOE_OK: return "ok";
    case VMOE_ERR_INVALID_ARG: return "invalid argument";
    case VMOE_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case VMOE_ERR_CUDA: return "CUDA error";
    case VMOE_ERR_NCCL: return "NCCL error";
    case VMOE_ERR_TIMEOUT: return "device wait timed out";
    case VMOE_ERR_DEVICE_STATUS: return "device reported an error";
    case VMOE_ERR_NOT_READY: return "weights not set";
    case VMOE_ERR_WORKSPACE: return "workspace too small or misaligned";
    default: return "unknown status";
  }
}

const char* vmoe_last_error(const vmoe_handle* h) { return h ? h->err.c_str() : ""; }

const char* vmoe_stage_name(int stage) {
  return (stage >= 0 && stage < kStages) ? kStageNames[stage] : "";
}

int vmoe_create(const vmoe_config* cfg, int device, vmoe_handle** out) {
  if (!cfg || !out) return VMOE_ERR_INVALID_ARG;
  *out = nullptr;
  char why[256];
  const int v = validate_config(cfg, why, sizeof(why));
  if (v != VMOE_OK) {
    fprintf(stderr, "vmoe_create: %s\n", why);
    return v;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    fprintf(stderr, "vmoe_create: CUDA device %d is not available\n", device);
    return VMOE_ERR_CUDA;
  }
  vmoe_handle* h = new (std::nothrow) vmoe_handle();
  if (!h) return VMOE_ERR_CUDA;
  h->cfg = *cfg;
  h->device = device;
  h->dtype = cfg->dtype;
  h->H = cfg->hidden;
  h->I = cfg->inter;
  h->E = cfg->num_experts;
  h->E_local = cfg->num_experts;
  h->K = cfg->top_k;
  if (h->dtype == kBF16) {
    h->Ipad = round_up(h->I, kGateUpInterleave);
    h->Hpad = round_up(h->H, kDownTileN);
    const char* pair = getenv("VMOE_PAIR_GEMM");  // "0" selects the single-CTA GEMMs
    h->tile_rows = (pair && pair[0] == '0') ? kTileM : 2 * kTileM;
  } else {
    h->Ipad = h->I;
    h->Hpad = h->H;
  }
  DeviceGuard g(device);
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (h->dtype == kBF16) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0) {
      fprintf(stderr, "vmoe_create: the bf16 path needs an sm_100 GPU (got sm_%d%d)\n", major,
              minor);
      delete h;
      return VMOE_ERR_UNSUPPORTED_SHAPE;
    }
  }
  cudaError_t e = cudaMalloc(&h->status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(h->status, 0, sizeof(int));
  if (e != cudaSuccess) {
    fprintf(stderr, "vmoe_create: %s\n", cudaGetErrorString(e));
    vmoe_destroy(h);
    return VMOE_ERR_CUDA;
  }
  *out = h;
  return VMOE_OK;
}

int vmoe_destroy(vmoe_handle* h) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  {
    DeviceGuard g(h->device);
    free_weights(h);
    for (P2PChannel& c : h->p2p) {
      for (size_t r = 0; r < c.peers.size(); ++r)
        if (static_cast<int>(r) != h->ep_rank && c.peers[r]) cudaIpcCloseMemHandle(c.peers[r]);
      if (c.region) cudaFree(c.region);
      if (c.peers_dev) cudaFree(c.peers_dev);
      if (c.block_counter) cudaFree(c.block_counter);
    }
    for (int i = 0; i < kMaxChunks; ++i) {
      if (h->p2p_streams[i]) cudaStreamDestroy(h->p2p_streams[i]);
      if (h->p2p_done[i]) cudaEventDestroy(h->p2p_done[i]);
      if (h->p2p_gemm_done[i]) cudaEventDestroy(h->p2p_gemm_done[i]);
      if (h->p2p_sent[i]) cudaEventDestroy(h->p2p_sent[i]);
    }
    if (h->p2p_start) cudaEventDestroy(h->p2p_start);
    for (int i = 0; i < kMaxHostChunks; ++i) {
      if (h->host_in_ev[i]) cudaEventDestroy(h->host_in_ev[i]);
      if (h->host_comp_ev[i]) cudaEventDestroy(h->host_comp_ev[i]);
    }
    if (h->host_start) cudaEventDestroy(h->host_start);
    if (h->host_out_done) cudaEventDestroy(h->host_out_done);
    if (h->host_in) cudaStreamDestroy(h->host_in);
    if (h->host_out) cudaStreamDestroy(h->host_out);
    if (h->status) cudaFree(h->status);
    if (h->ln_w) cudaFree(h->ln_w);
    if (h->ln_b) cudaFree(h->ln_b);
    if (h->w_dT) cudaFree(h->w_dT);
    if (h->w_guT) cudaFree(h->w_guT);
    if (h->w_rT) cudaFree(h->w_rT);
    for (cudaEvent_t ev : h->prof_ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : h->bprof_ev) cudaEventDestroy(ev);
  }
  delete h;
  return VMOE_OK;
}

namespace {
// Transposed copies of the packed (FlyLoRA-folded) weights for the backward GEMMs.
int make_training_copies(vmoe_handle* h, cudaStream_t s) {
  const int64_t E = h->E, H = h->H, Hpad = h->Hpad, Ipad = h->Ipad;
  h->Ipad2 = round_up(Ipad, 256);
  h->Epad64 = round_up(E, 64);
  int rc;
  if (!h->w_dT && (rc = alloc(h, &h->w_dT, E * h->Ipad2 * Hpad * 2, "W_d^T")) != VMOE_OK) return rc;
  if (!h->w_guT && (rc = alloc(h, &h->w_guT, E * Hpad * 2 * Ipad * 2, "gate|up^T")) != VMOE_OK)
    return rc;
  if (!h->w_rT && (rc = alloc(h, &h->w_rT, Hpad * h->Epad64 * 2, "W_r^T")) != VMOE_OK) return rc;
  cudaError_t e = launch_transpose_bf16(h->w_d, Hpad, Ipad, Ipad, Hpad * Ipad, static_cast<int>(E),
                                        h->w_dT, h->Ipad2, Hpad, h->Ipad2 * Hpad, nullptr, s);
  if (e == cudaSuccess)
    e = launch_transpose_bf16(h->w_g, 2 * Ipad, H, H, 2 * Ipad * H, static_cast<int>(E), h->w_guT,
                              Hpad, 2 * Ipad, Hpad * 2 * Ipad, nullptr, s);
  if (e == cudaSuccess)
    e = launch_transpose_bf16(h->w_r, E, H, H, 0, 1, h->w_rT, Hpad, h->Epad64, 0, nullptr, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "weight transposes");
  char why[256];
  if (!make_tmap_bf16(&h->map_wdT, h->w_dT, E * h->Ipad2, Hpad, Hpad, 128, why, sizeof(why)) ||
      !make_tmap_bf16(&h->map_guT, h->w_guT, E * Hpad, 2 * Ipad, 2 * Ipad, 128, why, sizeof(why)) ||
      !make_tmap_bf16(&h->map_wrT, h->w_rT, Hpad, h->Epad64, h->Epad64, 256, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "backward weight tensor maps: %s", why);
  return VMOE_OK;
}

// The LayerNorm fold of the tensor-core router (W_r * ln_w, its row sums, b_r + W_r ln_b);
// the CUDA-core router needs none.  Runs after the weights or the norm change.
int refold_norm(vmoe_handle* h, cudaStream_t s) {
  h->ln_ready = false;
  if (h->dtype == kBF16 && h->router_bn > 0) {
    const int64_t E = h->E, H = h->H;
    int rc;
    if (!h->w_r_ln && (rc = alloc(h, &h->w_r_ln, E * H * 2, "folded router weight")) != VMOE_OK)
      return rc;
    if (!h->b_r_ln && (rc = alloc(h, &h->b_r_ln, E * 4, "folded router bias")) != VMOE_OK) return rc;
    if (!h->c_ln && (rc = alloc(h, &h->c_ln, E * 4, "folded router sums")) != VMOE_OK) return rc;
    cudaError_t e = launch_fold_router_ln(h->w_r, h->b_r, h->ln_w, h->ln_b, static_cast<int>(E),
                                          static_cast<int>(H), h->w_r_ln, h->b_r_ln, h->c_ln, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "router LayerNorm fold");
    char why[256];
    if (!make_tmap_bf16(&h->map_wr_ln, h->w_r_ln, E, H, H, static_cast<uint32_t>(h->router_bn),
                        why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "folded router tensor map: %s", why);
  }
  h->ln_ready = true;
  return VMOE_OK;
}
}  // namespace

int vmoe_set_weights(vmoe_handle* h, const vmoe_weights* w, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  if (!w) return fail(h, VMOE_ERR_INVALID_ARG, "weights is NULL");
  if ((!w->router_w && !h->dense) || !w->gate_w || !w->up_w || !w->down_w)
    return fail(h, VMOE_ERR_INVALID_ARG, "router_w, gate_w, up_w and down_w are required");
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  free_weights(h);
  const int64_t E = h->E, H = h->H, I = h->I, Ipad = h->Ipad, Hpad = h->Hpad;
  const int64_t El = h->E_local;  // experts held by this handle (E without expert parallelism)
  const size_t elt = dtype_bytes(h->dtype);
  const bool bf16 = h->dtype == kBF16;
  const int R = h->cfg.lora_rank;
  int rc;
  if ((rc = alloc(h, &h->w_r, E * H * elt, "router weight")) != VMOE_OK) return rc;
  if ((rc = alloc(h, &h->b_r, E * 4, "router bias")) != VMOE_OK) return rc;
  const int64_t gu_rows = bf16 ? 2 * Ipad : I;
  if ((rc = alloc(h, &h->w_g, El * gu_rows * H * elt, "gate weight")) != VMOE_OK) return rc;
  if ((rc = alloc(h, &h->b_g, El * gu_rows * 4, "gate bias")) != VMOE_OK) return rc;
  if (!bf16) {
    if ((rc = alloc(h, &h->w_u, El * I * H * elt, "up weight")) != VMOE_OK) return rc;
    if ((rc = alloc(h, &h->b_u, El * I * 4, "up bias")) != VMOE_OK) return rc;
  }
  if ((rc = alloc(h, &h->w_d, El * Hpad * Ipad * elt, "down weight")) != VMOE_OK) return rc;
  if ((rc = alloc(h, &h->b_d, El * Hpad * 4, "down bias")) != VMOE_OK) return rc;

  cudaError_t e;
  // router: plain copy of W_r, bias to fp32 (zeros for a dense handle)
  if (w->router_w)
    e = cudaMemcpyAsync(h->w_r, w->router_w, E * H * elt, cudaMemcpyDeviceToDevice, s);
  else
    e = cudaMemsetAsync(h->w_r, 0, E * H * elt, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "router weight copy");
  {
    PackBiasArgs b{h->dtype, w->router_b, nullptr, nullptr, nullptr, 0, 0.f,
                   static_cast<int>(1), static_cast<int>(E), h->b_r, static_cast<int>(E), 0, 0};
    if ((e = launch_pack_bias(b, s)) != cudaSuccess) return cuda_fail(h, e, "router bias pack");
  }
  // gate / up with the FlyLoRA fold
  const bool lora_g = R > 0 && w->gate_lora_down_w && w->gate_lora_up_w;
  const bool lora_u = R > 0 && w->up_lora_down_w && w->up_lora_up_w;
  for (int which = 0; which < 2; ++which) {
    const bool lo = which == 0 ? lora_g : lora_u;
    PackArgs p{};
    p.dtype = h->dtype;
    p.src = which == 0 ? w->gate_w : w->up_w;
    p.lora_down = lo ? (which == 0 ? w->gate_lora_down_w : w->up_lora_down_w) : nullptr;
    p.lora_up = lo ? (which == 0 ? w->gate_lora_up_w : w->up_lora_up_w) : nullptr;
    p.R = lo ? R : 0;
    p.scaling = h->cfg.lora_scaling;
    p.E = static_cast<int>(El);
    p.O = static_cast<int>(I);
    p.Kin = static_cast<int>(H);
    p.Kpad = static_cast<int>(H);
    if (bf16) {
      p.dst = h->w_g;
      p.dst_rows_per_expert = static_cast<int>(2 * Ipad);
      p.interleave = kGateUpInterleave;
      p.which = which;
    } else {
      p.dst = which == 0 ? h->w_g : h->w_u;
      p.dst_rows_per_expert = static_cast<int>(I);
      p.interleave = 0;
      p.which = 0;
    }
    if ((e = launch_pack_weight(p, s)) != cudaSuccess) return cuda_fail(h, e, "gate/up pack");
    PackBiasArgs b{};
    b.dtype = h->dtype;
    b.b = which == 0 ? w->gate_b : w->up_b;
    b.lora_up = p.lora_up;
    b.lora_down_b = lo ? (which == 0 ? w->gate_lora_down_b : w->up_lora_down_b) : nullptr;
    b.lora_up_b = lo ? (which == 0 ? w->gate_lora_up_b : w->up_lora_up_b) : nullptr;
    b.R = p.R;
    b.scaling = p.scaling;
    b.E = p.E;
    b.O = p.O;
    b.dst = bf16 ? h->b_g : (which == 0 ? h->b_g : h->b_u);
    b.dst_per_expert = p.dst_rows_per_expert;
    b.interleave = p.interleave;
    b.which = p.which;
    if ((e = launch_pack_bias(b, s)) != cudaSuccess) return cuda_fail(h, e, "gate/up bias pack");
  }
  // down projection, zero padded to [E, Hpad, Ipad]
  {
    PackArgs p{};
    p.dtype = h->dtype;
    p.src = w->down_w;
    p.E = static_cast<int>(El);
    p.O = static_cast<int>(H);
    p.Kin = static_cast<int>(I);
    p.Kpad = static_cast<int>(Ipad);
    p.dst = h->w_d;
    p.dst_rows_per_expert = static_cast<int>(Hpad);
    if ((e = launch_pack_weight(p, s)) != cudaSuccess) return cuda_fail(h, e, "down pack");
    PackBiasArgs b{};
    b.dtype = h->dtype;
    b.b = w->down_b;
    b.E = p.E;
    b.O = p.O;
    b.dst = h->b_d;
    b.dst_per_expert = static_cast<int>(Hpad);
    if ((e = launch_pack_bias(b, s)) != cudaSuccess) return cuda_fail(h, e, "down bias pack");
  }
  if (bf16) {
    char why[256];
    h->router_bn = tc_router_width(static_cast<int>(E));
    if (h->router_bn &&
        !make_tmap_bf16(&h->map_wr, h->w_r, E, H, H, static_cast<uint32_t>(h->router_bn), why,
                        sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "router tensor map: %s", why);
    // B tiles: 256 rows per CTA, or 128 per CTA of a pair
    const uint32_t b_box = h->tile_rows == kTileM ? 256u : 128u;
    if (!make_tmap_bf16(&h->map_wgu, h->w_g, El * 2 * Ipad, H, H, b_box, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "gate/up tensor map: %s", why);
    if (!make_tmap_bf16(&h->map_wd, h->w_d, El * Hpad, Ipad, Ipad, b_box, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "down tensor map: %s", why);
  }
  h->ready = true;
  if (h->ln_w && (rc = refold_norm(h, s)) != VMOE_OK) return rc;
  if (h->training && (rc = make_training_copies(h, s)) != VMOE_OK) return rc;
  h->err.clear();
  return VMOE_OK;
}

int vmoe_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes) {
  if (!h || !bytes || tokens < 0) return VMOE_ERR_INVALID_ARG;
  *bytes = make_plan(h, tokens).total;
  return VMOE_OK;
}

int vmoe_workspace_layout(const vmoe_handle* h, int64_t tokens, vmoe_ws_layout* out) {
  if (!h || !out || tokens < 0) return VMOE_ERR_INVALID_ARG;
  const Plan p = make_plan(h, tokens);
  out->slot_of = p.slot;
  out->expert_offsets = p.offs;
  out->num_tiles = p.ntiles;
  out->x_perm = p.xp;
  out->h = p.h;
  out->y = p.y;
  out->max_rows = p.max_rows;
  out->h_ld = h->Ipad;
  out->y_ld = h->Hpad;
  out->total = p.total;
  return VMOE_OK;
}

int vmoe_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out, float* router_logits,
                 int32_t* topk_idx, float* topk_w, int32_t* expert_counts, float* aux_loss,
                 void* workspace, size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (h->ep_size > 1)
    return fail(h, VMOE_ERR_INVALID_ARG,
                "an expert-parallel handle runs through vmoe_ep_route/experts/combine");
  if (tokens < 0) return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be >= 0 (got %lld)",
                              static_cast<long long>(tokens));
  const int64_t E = h->E, K = h->K, H = h->H, T = tokens;
  if (T * K + E * kTileM >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "tokens * top_k too large (%lld)",
                static_cast<long long>(T * K));
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (T == 0) {
    // An empty batch: no output rows; the reference's mean over zero tokens makes aux NaN.
    if (aux_loss) {
      const float nan = __builtin_nanf("");
      if ((e = cudaMemcpyAsync(aux_loss, &nan, 4, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_fail(h, e, "aux write");
    }
    if (expert_counts && (e = cudaMemsetAsync(expert_counts, 0, E * 4, s)) != cudaSuccess)
      return cuda_fail(h, e, "counts write");
    return VMOE_OK;
  }
  if (!x || !out) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const Plan p = make_plan(h, T);
  if (!workspace || workspace_bytes < p.total)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", p.total,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");

  const bool prof = h->prof_count < h->prof_slots;
  const int rc = forward_batch(h, x, T, out, router_logits, topk_idx, topk_w, expert_counts,
                               aux_loss, static_cast<char*>(workspace), p, s, prof, nullptr);
  if (rc == VMOE_OK && prof) ++h->prof_count;
  return rc;
}

int vmoe_set_norm(vmoe_handle* h, const void* ln_weight, const void* ln_bias, float eps,
                  void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  if (h->dense || h->ep_size > 1)
    return fail(h, VMOE_ERR_INVALID_ARG, "the fused pre-norm takes a single-GPU MoE handle");
  if (!(eps >= 0.f) || eps > 1.f)
    return fail(h, VMOE_ERR_INVALID_ARG, "eps must be in [0, 1] (got %g)", static_cast<double>(eps));
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t H = h->H;
  int rc;
  if (!h->ln_w && (rc = alloc(h, &h->ln_w, H * 4, "LayerNorm weight")) != VMOE_OK) return rc;
  if (!h->ln_b && (rc = alloc(h, &h->ln_b, H * 4, "LayerNorm bias")) != VMOE_OK) return rc;
  cudaError_t e = launch_to_f32(h->dtype, ln_weight, H, 1.f, h->ln_w, s);
  if (e == cudaSuccess) e = launch_to_f32(h->dtype, ln_bias, H, 0.f, h->ln_b, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "LayerNorm parameters");
  h->ln_eps = eps;
  h->ln_ready = false;
  return h->ready ? refold_norm(h, s) : VMOE_OK;
}

int vmoe_forward_residual(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                          float* router_logits, int32_t* topk_idx, float* topk_w,
                          int32_t* expert_counts, float* aux_loss, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (!h->ln_ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_norm has not been called");
  if (tokens < 0) return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be >= 0 (got %lld)",
                              static_cast<long long>(tokens));
  const int64_t E = h->E, K = h->K, T = tokens;
  if (T * K + E * kTileM >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "tokens * top_k too large (%lld)",
                static_cast<long long>(T * K));
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (T == 0) {
    if (aux_loss) {
      const float nan = __builtin_nanf("");
      if ((e = cudaMemcpyAsync(aux_loss, &nan, 4, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_fail(h, e, "aux write");
    }
    if (expert_counts && (e = cudaMemsetAsync(expert_counts, 0, E * 4, s)) != cudaSuccess)
      return cuda_fail(h, e, "counts write");
    return VMOE_OK;
  }
  if (!x || !out) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const Plan p = make_plan(h, T);
  if (!workspace || workspace_bytes < p.total)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", p.total,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const bool prof = h->prof_count < h->prof_slots;
  const int rc = forward_batch(h, x, T, out, router_logits, topk_idx, topk_w, expert_counts,
                               aux_loss, static_cast<char*>(workspace), p, s, prof, nullptr, true);
  if (rc == VMOE_OK && prof) ++h->prof_count;
  return rc;
}

// ---- forward on host buffers: chunked copy-in / compute / copy-out pipeline -------------
namespace {

struct HostPlan {
  int chunks = 1;
  int64_t chunk_tokens = 0;
  size_t x = 0, out = 0, small = 0, small_stride = 0, psum_off = 0, aux = 0, fwd = 0, total = 0;
  // chunks > 1: the batch's routing tables, one chunk's routing scratch, the carry state
  // (two of each: chunk c reads c-1's) and a ring of two chunk buffers for x_perm / h / y
  int nblk = 0;
  int64_t ring_rows = 0;
  size_t idx = 0, w = 0, slot = 0, hist = 0, psum = 0, excl = 0, offs = 0, comp = 0, tiles = 0,
         ntiles = 0, ccnt = 0, clist = 0, xp = 0, hb = 0, y = 0;
};

// Workspace: x and out of the whole batch on the device and per-chunk expert counts and
// probability sums (for the aux loss of the whole batch).  One chunk: that chunk's forward
// workspace.  Several: the carry pipeline's tables and buffers (HostPlan).  With a token
// capacity the batch is one chunk (the capacity applies to the batch as a whole).
HostPlan make_host_plan(const vmoe_handle* h, int64_t T, int chunks) {
  HostPlan hp;
  if (chunks <= 0) {  // automatic: chunks of at least 8192 tokens, at most 8 of them
    const int64_t a = T / 8192;
    chunks = a < 1 ? 1 : (a > 8 ? 8 : static_cast<int>(a));
  }
  if (chunks > kMaxHostChunks) chunks = kMaxHostChunks;
  if (h->cfg.capacity > 0) chunks = 1;
  int64_t ct = round_up((T + chunks - 1) / chunks, kTileM);
  if (ct < kTileM) ct = kTileM;
  hp.chunk_tokens = ct;
  hp.chunks = T > 0 ? static_cast<int>((T + ct - 1) / ct) : 1;
  const size_t elt = dtype_bytes(h->dtype);
  const size_t row = static_cast<size_t>(h->H) * elt;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  hp.x = take(static_cast<size_t>(T) * row);
  hp.out = take(static_cast<size_t>(T) * row);
  hp.small_stride = round_up(8 * h->E, 256);
  hp.psum_off = 4 * h->E;
  hp.small = take(hp.small_stride * hp.chunks);
  hp.aux = take(4);
  if (hp.chunks == 1) {
    hp.fwd = take(make_plan(h, T < ct ? T : ct).total);
  } else {
    const int64_t E = h->E, K = h->K, tr = h->tile_rows;
    hp.nblk = static_cast<int>(ct / kTileM);
    // a chunk's segments: its ct*K new rows plus up to tr-1 carried-in rows per expert, each
    // segment rounded up to whole tiles
    hp.ring_rows = round_up(ct * K + 2 * E * (tr - 1), tr);
    hp.idx = take(static_cast<size_t>(T) * K * 4);
    hp.w = take(static_cast<size_t>(T) * K * 4);
    hp.slot = take(static_cast<size_t>(T) * K * 4);
    hp.hist = take(static_cast<size_t>(hp.nblk) * E * 4);
    hp.psum = take(static_cast<size_t>(hp.nblk) * E * 4);
    hp.excl = take(static_cast<size_t>(hp.nblk) * E * 4);
    hp.offs = take((E + 1) * 4);
    hp.comp = take(E * 4);
    hp.tiles = take(static_cast<size_t>(hp.ring_rows / tr) * 4);
    hp.ntiles = take(4);
    hp.ccnt = take(2 * E * 4);
    hp.clist = take(static_cast<size_t>(2) * E * kCarryCap * 4);
    hp.xp = take(2 * static_cast<size_t>(hp.ring_rows) * row);
    hp.hb = take(2 * static_cast<size_t>(hp.ring_rows) * h->Ipad * elt);
    hp.y = take(2 * static_cast<size_t>(hp.ring_rows) * h->Hpad * elt);
  }
  hp.total = off;
  return hp;
}

// Chunks c = 0..C-1 of the host-buffer forward with carried rows.  Chunk c routes its
// tokens, computes the whole tiles of its expert segments (the rows carried in from c-1
// first) in ring buffer c % 2 and carries each segment's remainder to chunk c+1; once chunk
// c's GEMMs are done every row of chunk c-1 has been computed, so c-1 is combined and
// copied out while c+1 runs.  The last two chunks carry nothing out (they pad their last
// tiles instead), so each is copied out right after its own GEMMs and only one chunk's
// copy-out is left after the last GEMM.  Each row's GEMM output and each token's combine
// are the same as in one forward of the whole batch, so out is bit-identical to
// vmoe_forward.
int host_chunks_with_carry(vmoe_handle* h, int64_t T, const HostPlan& hp, char* ws,
                           void* out_host, cudaStream_t s) {
  const int64_t E = h->E, K = h->K, H = h->H, tr = h->tile_rows;
  const size_t elt = dtype_bytes(h->dtype), row = static_cast<size_t>(H) * elt;
  const int C = hp.chunks;
  int32_t* idx = reinterpret_cast<int32_t*>(ws + hp.idx);
  float* tw = reinterpret_cast<float*>(ws + hp.w);
  int* slot = reinterpret_cast<int*>(ws + hp.slot);
  int* hist = reinterpret_cast<int*>(ws + hp.hist);
  float* psum = reinterpret_cast<float*>(ws + hp.psum);
  int* excl = reinterpret_cast<int*>(ws + hp.excl);
  int* offs = reinterpret_cast<int*>(ws + hp.offs);
  int* comp = reinterpret_cast<int*>(ws + hp.comp);
  int* tiles = reinterpret_cast<int*>(ws + hp.tiles);
  int* ntiles = reinterpret_cast<int*>(ws + hp.ntiles);
  int* ccnt = reinterpret_cast<int*>(ws + hp.ccnt);    // [2][E]
  int* clist = reinterpret_cast<int*>(ws + hp.clist);  // [2][E][kCarryCap]
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  auto no_mark = []() {};
  auto chunk_range = [&](int c, int64_t* t0, int64_t* tc) {
    *t0 = c * hp.chunk_tokens;
    *tc = (T - *t0) < hp.chunk_tokens ? (T - *t0) : hp.chunk_tokens;
  };
  // combine chunk c (all its rows computed) and copy it out
  auto finish = [&](int c) -> int {
    int64_t t0, tc;
    chunk_range(c, &t0, &tc);
    int r = check(launch_combine(h->dtype, ws + hp.y, h->Hpad, idx + t0 * K, tw + t0 * K,
                                 slot + t0 * K, tc, static_cast<int>(H), static_cast<int>(K),
                                 ws + hp.out + t0 * row, nullptr, s),
                  "combine");
    if (r != VMOE_OK) return r;
    cudaError_t e;
    if ((e = cudaEventRecord(h->host_comp_ev[c], s)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(h->host_out, h->host_comp_ev[c], 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(static_cast<char*>(out_host) + t0 * row, ws + hp.out + t0 * row,
                             tc * row, cudaMemcpyDeviceToHost, h->host_out)) != cudaSuccess)
      return cuda_fail(h, e, "copy out");
    return VMOE_OK;
  };
  cudaError_t e = cudaMemsetAsync(ccnt, 0, 2 * E * 4, s);  // nothing carried into chunk 0
  if (e != cudaSuccess) return cuda_fail(h, e, "carry counts");
  int rc, finished = 0;
  for (int c = 0; c < C; ++c) {
    int64_t t0, tc;
    chunk_range(c, &t0, &tc);
    const int cur = c & 1, prev = cur ^ 1;
    const int64_t slot_base = cur * hp.ring_rows;
    char* xp = ws + hp.xp + cur * hp.ring_rows * row;
    char* hb = ws + hp.hb + cur * hp.ring_rows * h->Ipad * elt;
    char* yb = ws + hp.y + cur * hp.ring_rows * h->Hpad * elt;
    char* small = ws + hp.small + c * hp.small_stride;
    int* counts = reinterpret_cast<int*>(small);
    const char* xc = ws + hp.x + t0 * row;
    if ((e = cudaStreamWaitEvent(s, h->host_in_ev[c], 0)) != cudaSuccess)
      return cuda_fail(h, e, "wait");
    const int nblk = static_cast<int>((tc + kTileM - 1) / kTileM);
    if ((rc = run_router(h, xc, tc, nullptr, idx + t0 * K, tw + t0 * K, hist, psum, nullptr,
                         s)) != VMOE_OK)
      return rc;
    if ((rc = check(launch_scan_blocks(hist, psum, nblk, static_cast<int>(E), excl, counts,
                                       reinterpret_cast<float*>(small + hp.psum_off), s),
                    "scan")) != VMOE_OK)
      return rc;
    if ((rc = check(launch_plan_carry(counts, ccnt + prev * E, static_cast<int>(E), c >= C - 2,
                                      static_cast<int>(tr), offs, comp, ccnt + cur * E, tiles,
                                      ntiles, s),
                    "plan")) != VMOE_OK)
      return rc;
    if (c > 0 &&
        (rc = check(launch_carry_rows(h->dtype, ws + hp.x, static_cast<int>(H),
                                      static_cast<int>(E), static_cast<int>(K),
                                      clist + prev * E * kCarryCap, ccnt + prev * E, offs, xp, H,
                                      slot_base, slot, h->status, s),
                    "carried rows")) != VMOE_OK)
      return rc;
    if ((rc = check(launch_dispatch_carry(h->dtype, xc, idx + t0 * K, excl, offs, tc,
                                          static_cast<int>(H), static_cast<int>(E),
                                          static_cast<int>(K), slot + t0 * K, xp, H,
                                          ccnt + prev * E, comp, clist + cur * E * kCarryCap, t0,
                                          slot_base, h->status, s),
                    "dispatch")) != VMOE_OK)
      return rc;
    if ((rc = run_expert_gemms(h, xp, hp.ring_rows, tiles, ntiles, hb, yb, h->Hpad, s, no_mark,
                               check)) != VMOE_OK)
      return rc;
    // every row of chunks < c is computed now, and of chunk c too when it carried nothing
    const int upto = c >= C - 2 ? c : c - 1;
    while (finished <= upto)
      if ((rc = finish(finished++)) != VMOE_OK) return rc;
  }
  return VMOE_OK;
}

void CUDART_CB write_nan(void* p) { *static_cast<float*>(p) = __builtin_nanf(""); }

int ensure_host_streams(vmoe_handle* h) {
  if (h->host_in) return VMOE_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&h->host_in, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->host_out, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->host_start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->host_out_done, cudaEventDisableTiming);
  for (int c = 0; c < kMaxHostChunks && e == cudaSuccess; ++c) {
    e = cudaEventCreateWithFlags(&h->host_in_ev[c], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->host_comp_ev[c], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    // leave the handle as it was so that a later call retries
    if (h->host_in) cudaStreamDestroy(h->host_in);
    if (h->host_out) cudaStreamDestroy(h->host_out);
    h->host_in = h->host_out = nullptr;
    return cuda_fail(h, e, "host copy streams");
  }
  return VMOE_OK;
}

}  // namespace

int vmoe_forward_host_workspace_size(const vmoe_handle* h, int64_t tokens, int chunks,
                                     size_t* bytes) {
  if (!h || !bytes || tokens < 0) return VMOE_ERR_INVALID_ARG;
  *bytes = make_host_plan(h, tokens, chunks).total;
  return VMOE_OK;
}

int vmoe_forward_host(vmoe_handle* h, const void* x_host, int64_t tokens, void* out_host,
                      float* aux_loss_host, int chunks, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (h->ep_size > 1 || h->dense)
    return fail(h, VMOE_ERR_INVALID_ARG, "vmoe_forward_host takes a single-GPU MoE handle");
  if (tokens < 0) return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be >= 0 (got %lld)",
                              static_cast<long long>(tokens));
  const int64_t E = h->E, K = h->K, T = tokens;
  if (T * K + E * kTileM >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "tokens * top_k too large (%lld)",
                static_cast<long long>(T * K));
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (T == 0) {  // as vmoe_forward: no rows, aux NaN (written in stream order)
    if (aux_loss_host && (e = cudaLaunchHostFunc(s, write_nan, aux_loss_host)) != cudaSuccess)
      return cuda_fail(h, e, "aux write");
    return VMOE_OK;
  }
  if (!x_host || !out_host) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if (chunks < 0 || chunks > kMaxHostChunks)
    return fail(h, VMOE_ERR_INVALID_ARG, "chunks must be in [0, %d] (got %d)", kMaxHostChunks,
                chunks);
  const HostPlan hp = make_host_plan(h, T, chunks);
  if (!workspace || workspace_bytes < hp.total)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", hp.total,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  int rc = ensure_host_streams(h);
  if (rc != VMOE_OK) return rc;

  char* ws = static_cast<char*>(workspace);
  const size_t row = static_cast<size_t>(h->H) * dtype_bytes(h->dtype);
  const int C = hp.chunks;
  float* aux_dev = reinterpret_cast<float*>(ws + hp.aux);
  // the copy-in of this call may overwrite x only after the caller's earlier work on s
  if ((e = cudaEventRecord(h->host_start, s)) != cudaSuccess) return cuda_fail(h, e, "event");
  if ((e = cudaStreamWaitEvent(h->host_in, h->host_start, 0)) != cudaSuccess)
    return cuda_fail(h, e, "wait");
  // every exit after this point joins the copy streams into s
  auto join = [&](int code) {
    cudaEventRecord(h->host_out_done, h->host_out);
    cudaStreamWaitEvent(s, h->host_out_done, 0);
    cudaEventRecord(h->host_out_done, h->host_in);
    cudaStreamWaitEvent(s, h->host_out_done, 0);
    return code;
  };
  for (int c = 0; c < C; ++c) {
    const int64_t t0 = c * hp.chunk_tokens;
    const int64_t tc = (T - t0) < hp.chunk_tokens ? (T - t0) : hp.chunk_tokens;
    if ((e = cudaMemcpyAsync(ws + hp.x + t0 * row, static_cast<const char*>(x_host) + t0 * row,
                             tc * row, cudaMemcpyHostToDevice, h->host_in)) != cudaSuccess ||
        (e = cudaEventRecord(h->host_in_ev[c], h->host_in)) != cudaSuccess)
      return join(cuda_fail(h, e, "copy in"));
  }
  if (C == 1) {
    if ((e = cudaStreamWaitEvent(s, h->host_in_ev[0], 0)) != cudaSuccess)
      return join(cuda_fail(h, e, "wait"));
    rc = forward_batch(h, ws + hp.x, T, ws + hp.out, nullptr, nullptr, nullptr, nullptr, aux_dev,
                       ws + hp.fwd, make_plan(h, T), s, false, nullptr);
    if (rc != VMOE_OK) return join(rc);
    if ((e = cudaEventRecord(h->host_comp_ev[0], s)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(h->host_out, h->host_comp_ev[0], 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(out_host, ws + hp.out, T * row, cudaMemcpyDeviceToHost,
                             h->host_out)) != cudaSuccess)
      return join(cuda_fail(h, e, "copy out"));
  } else if ((rc = host_chunks_with_carry(h, T, hp, ws, out_host, s)) != VMOE_OK) {
    return join(rc);
  }
  if (aux_loss_host) {
    if (C > 1) {  // the loss of the whole batch from every chunk's counts and sums
      if ((e = launch_aux_merge_ws(ws + hp.small, hp.small_stride, 0, hp.psum_off, C, T,
                                   static_cast<int>(E), static_cast<int>(K), aux_dev, s)) !=
          cudaSuccess)
        return join(cuda_fail(h, e, "aux merge"));
      ++h->last_launches;
    }
    if ((e = cudaMemcpyAsync(aux_loss_host, aux_dev, 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
      return join(cuda_fail(h, e, "aux copy"));
  }
  return join(VMOE_OK);
}

int vmoe_create_ep(const vmoe_config* cfg, int device, int ep_size, int ep_rank,
                   vmoe_handle** out) {
  if (!cfg || !out) return VMOE_ERR_INVALID_ARG;
  *out = nullptr;
  if (ep_size < 1 || ep_rank < 0 || ep_rank >= ep_size || cfg->num_experts % ep_size) {
    fprintf(stderr, "vmoe_create_ep: need 0 <= ep_rank < ep_size and num_experts %% ep_size == 0"
            " (E=%d, ep_size=%d, ep_rank=%d)\n", cfg->num_experts, ep_size, ep_rank);
    return VMOE_ERR_INVALID_ARG;
  }
  if (cfg->capacity != 0) {
    fprintf(stderr, "vmoe_create_ep: capacity is not supported with expert parallelism\n");
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  if (cfg->dtype == VMOE_BF16 && cfg->hidden % kDownTileN) {
    fprintf(stderr, "vmoe_create_ep: bf16 expert parallelism needs hidden %% %d == 0\n",
            kDownTileN);
    return VMOE_ERR_UNSUPPORTED_SHAPE;
  }
  vmoe_handle* h = nullptr;
  const int rc = vmoe_create(cfg, device, &h);
  if (rc != VMOE_OK) return rc;
  h->ep_size = ep_size;
  h->ep_rank = ep_rank;
  h->E_local = cfg->num_experts / ep_size;
  *out = h;
  return VMOE_OK;
}

int vmoe_ep_workspace_size(const vmoe_handle* h, int64_t tokens, int64_t recv_rows_cap,
                           size_t* bytes) {
  if (!h || !bytes || tokens < 0 || recv_rows_cap < 0) return VMOE_ERR_INVALID_ARG;
  *bytes = make_ep_plan(h, tokens, recv_rows_cap).total;
  return VMOE_OK;
}

namespace {
int ep_common_checks(vmoe_handle* h, void* workspace, size_t workspace_bytes, size_t need) {
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (!workspace || workspace_bytes < need)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", need,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  return VMOE_OK;
}
}  // namespace

int vmoe_ep_route(vmoe_handle* h, const void* x, int64_t tokens, void* send_rows,
                  int32_t* expert_counts, float* router_logits, float* aux_loss, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  const int64_t E = h->E, K = h->K, H = h->H, T = tokens;
  if (T < 0 || T * K + E >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_INVALID_ARG, "bad token count %lld", static_cast<long long>(T));
  if (!expert_counts) return fail(h, VMOE_ERR_INVALID_ARG, "expert_counts is required");
  const EpPlan p = make_ep_plan(h, T, 0);
  int rc = ep_common_checks(h, workspace, workspace_bytes, p.total);
  if (rc != VMOE_OK) return rc;
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (T == 0) {
    if ((e = cudaMemsetAsync(expert_counts, 0, E * 4, s)) != cudaSuccess)
      return cuda_fail(h, e, "counts write");
    if (aux_loss) {
      const float nan = __builtin_nanf("");
      if ((e = cudaMemcpyAsync(aux_loss, &nan, 4, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_fail(h, e, "aux write");
    }
    return VMOE_OK;
  }
  if (!x || !send_rows) return fail(h, VMOE_ERR_INVALID_ARG, "x and send_rows are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send_rows)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and send_rows must be 16-byte aligned");
  char* ws = static_cast<char*>(workspace);
  int32_t* idx = reinterpret_cast<int32_t*>(ws + p.idx);
  float* tw = reinterpret_cast<float*>(ws + p.w);
  int* hist = reinterpret_cast<int*>(ws + p.hist);
  float* psum = reinterpret_cast<float*>(ws + p.psum);
  int* excl = reinterpret_cast<int*>(ws + p.excl);
  int* counts = reinterpret_cast<int*>(ws + p.counts);
  float* psum_tot = reinterpret_cast<float*>(ws + p.psum_tot);
  int* offs = reinterpret_cast<int*>(ws + p.offs);
  float* aux = aux_loss ? aux_loss : reinterpret_cast<float*>(ws + p.aux);
  int* slot = reinterpret_cast<int*>(ws + p.slot);
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  if ((rc = run_router(h, x, T, router_logits, idx, tw, hist, psum, nullptr, s)) != VMOE_OK)
    return rc;
  if ((rc = check(launch_scan_blocks(hist, psum, p.nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s), "scan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K), 0,
                              1, offs, nullptr, nullptr, aux, expert_counts, s), "plan")) != VMOE_OK)
    return rc;
  return check(launch_dispatch(h->dtype, x, idx, excl, offs, T, static_cast<int>(H),
                               static_cast<int>(E), static_cast<int>(K), 0, slot, send_rows, H,
                               h->status, nullptr, s), "dispatch");
}

int vmoe_ep_experts(vmoe_handle* h, const void* recv_rows, int64_t recv_rows_cap,
                    const int32_t* tile_expert, const int32_t* num_tiles, void* out_rows,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (recv_rows_cap < 0 || recv_rows_cap % h->tile_rows)
    return fail(h, VMOE_ERR_INVALID_ARG, "recv_rows_cap must be a multiple of %d (got %lld)",
                h->tile_rows, static_cast<long long>(recv_rows_cap));
  const EpPlan p = make_ep_plan(h, 0, recv_rows_cap);
  int rc = ep_common_checks(h, workspace, workspace_bytes, p.total);
  if (rc != VMOE_OK) return rc;
  if (recv_rows_cap == 0) return VMOE_OK;
  if (!recv_rows || !out_rows || !tile_expert || !num_tiles)
    return fail(h, VMOE_ERR_INVALID_ARG, "recv_rows, out_rows, tile_expert, num_tiles required");
  if ((reinterpret_cast<uintptr_t>(recv_rows) | reinterpret_cast<uintptr_t>(out_rows)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "row buffers must be 16-byte aligned");
  if (h->Hpad != h->H)
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "expert parallelism needs hidden %% %d == 0",
                kDownTileN);
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  auto mark = []() {};
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  return run_expert_gemms(h, const_cast<void*>(recv_rows), recv_rows_cap, tile_expert, num_tiles,
                          ws + p.h, out_rows, h->H, s, mark, check);
}

int vmoe_ep_combine(vmoe_handle* h, const void* back_rows, int64_t tokens, void* out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (tokens < 0) return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be >= 0");
  const EpPlan p = make_ep_plan(h, tokens, 0);
  int rc = ep_common_checks(h, workspace, workspace_bytes, p.total);
  if (rc != VMOE_OK) return rc;
  if (tokens == 0) return VMOE_OK;
  if (!back_rows || !out) return fail(h, VMOE_ERR_INVALID_ARG, "back_rows and out are required");
  if ((reinterpret_cast<uintptr_t>(back_rows) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "back_rows and out must be 16-byte aligned");
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const cudaError_t e = launch_combine(h->dtype, back_rows, h->H,
                                       reinterpret_cast<int32_t*>(ws + p.idx),
                                       reinterpret_cast<float*>(ws + p.w),
                                       reinterpret_cast<int*>(ws + p.slot), tokens,
                                       static_cast<int>(h->H), static_cast<int>(h->K), out,
                                       nullptr, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "combine");
  h->last_launches = 1;
  return VMOE_OK;
}

int vmoe_ep_p2p_setup(vmoe_handle* h, int64_t max_tokens, int chunks, void* ipc_handles) {
  if (!h || !ipc_handles || max_tokens < 0) return VMOE_ERR_INVALID_ARG;
  if (chunks < 1 || chunks > kMaxChunks)
    return fail(h, VMOE_ERR_INVALID_ARG, "chunks must be in [1, %d] (got %d)", kMaxChunks, chunks);
  if (!h->p2p.empty()) return fail(h, VMOE_ERR_INVALID_ARG, "vmoe_ep_p2p_setup was already called");
  if (h->dtype == kBF16 && h->Hpad != h->H)
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "bf16 expert parallelism needs hidden %% %d == 0",
                kDownTileN);
  const int64_t G = h->ep_size, E = h->E, K = h->K, El = h->E_local, H = h->H;
  const int64_t chunk_tokens = round_up((max_tokens + chunks - 1) / chunks, kTileM);
  const int64_t cap = round_up(G * chunk_tokens * K + El * (h->tile_rows - 1), h->tile_rows);
  if (cap >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "receive capacity of %lld rows is too large",
                static_cast<long long>(cap));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  // the bf16 CTA-pair GEMMs push their outputs to the source ranks up to 2 ranks; beyond,
  // the sources pull them in the combine (measured: with 4 ranks the down GEMM's epilogue
  // cannot keep enough remote stores in flight, and the pulling combine overlaps the next
  // chunk's GEMMs).  VMOE_EP_PUSH=1 / 0 forces either.  (The return address holds a 24-bit
  // row of the source's chunk and an 8-bit rank.)
  const char* pe = getenv("VMOE_EP_PUSH");
  const bool want_push = pe ? pe[0] == '1' : G <= 2;
  h->p2p_push = h->dtype == kBF16 && h->tile_rows == 2 * kTileM && want_push &&
                chunk_tokens * K < (static_cast<int64_t>(1) << 24) && G <= 256;
  h->p2p_sig_off = take(3 * G * 4);
  h->p2p_counts_off = take(G * E * 4);
  h->p2p_ret_off = h->p2p_push ? take(static_cast<size_t>(cap) * 8) : 0;
  h->p2p_recv_off = take(static_cast<size_t>(cap) * H * dtype_bytes(h->dtype));
  h->p2p_back_rows = chunk_tokens * K;
  if (h->p2p_push)
    h->p2p_back_off = take(static_cast<size_t>(h->p2p_back_rows) * H * dtype_bytes(h->dtype));
  else
    h->p2p_y_off = take(static_cast<size_t>(cap) * H * dtype_bytes(h->dtype));
  DeviceGuard g(h->device);
  h->p2p.resize(chunks);
  cudaError_t e = cudaSuccess;
  for (int c = 0; c < chunks && e == cudaSuccess; ++c) {
    P2PChannel& ch = h->p2p[c];
    e = cudaMalloc(&ch.region, off);
    if (e == cudaSuccess) e = cudaMemset(ch.region, 0, h->p2p_recv_off);
    if (e == cudaSuccess) e = cudaMalloc(&ch.block_counter, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ch.block_counter, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&ch.peers_dev, G * sizeof(char*));
    cudaIpcMemHandle_t mh;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mh, ch.region);
    if (e == cudaSuccess)
      memcpy(static_cast<char*>(ipc_handles) + static_cast<size_t>(c) * sizeof(mh), &mh, sizeof(mh));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->p2p_streams[c], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->p2p_done[c], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->p2p_gemm_done[c], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->p2p_sent[c], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->p2p_start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(h, e, "peer-memory region");
  h->p2p_cap_rows = cap;
  h->p2p_max_tokens = max_tokens;
  h->p2p_chunk_tokens = chunk_tokens;
  // VMOE_EP_RESERVE_SMS=n keeps n SMs out of the chunked GEMM grid for the NVLink transfer
  // kernels (off by default: on 2 GPUs it measured slower)
  h->p2p_reserve_sms = 0;
  if (const char* r = getenv("VMOE_EP_RESERVE_SMS")) h->p2p_reserve_sms = chunks > 1 ? atoi(r) : 0;
  if (h->p2p_reserve_sms < 0 || h->p2p_reserve_sms > h->num_sms / 2) h->p2p_reserve_sms = 0;
  return VMOE_OK;
}

int vmoe_ep_p2p_connect(vmoe_handle* h, const void* ipc_handles) {
  if (!h || !ipc_handles) return VMOE_ERR_INVALID_ARG;
  if (h->p2p.empty()) return fail(h, VMOE_ERR_NOT_READY, "vmoe_ep_p2p_setup has not been called");
  if (h->p2p_connected) return fail(h, VMOE_ERR_INVALID_ARG, "already connected");
  DeviceGuard g(h->device);
  const int G = h->ep_size, C = static_cast<int>(h->p2p.size());
  const char* bytes = static_cast<const char*>(ipc_handles);
  for (int c = 0; c < C; ++c) {
    P2PChannel& ch = h->p2p[c];
    ch.peers.assign(G, nullptr);
    for (int r = 0; r < G; ++r) {
      if (r == h->ep_rank) {
        ch.peers[r] = ch.region;
        continue;
      }
      cudaIpcMemHandle_t mh;
      memcpy(&mh, bytes + (static_cast<size_t>(r) * C + c) * sizeof(mh), sizeof(mh));
      void* p = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return cuda_fail(h, e, "cudaIpcOpenMemHandle of a peer region");
      ch.peers[r] = static_cast<char*>(p);
    }
    cudaError_t e = cudaMemcpy(ch.peers_dev, ch.peers.data(), G * sizeof(char*),
                               cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(h, e, "peer table");
  }
  h->p2p_connected = true;
  return VMOE_OK;
}

namespace {
size_t p2p_chunk_stride(const vmoe_handle* h) {
  return (make_p2p_plan(h, h->p2p_chunk_tokens).total + 255) & ~static_cast<size_t>(255);
}
}  // namespace

int vmoe_ep_p2p_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes) {
  if (!h || !bytes || tokens < 0) return VMOE_ERR_INVALID_ARG;
  if (h->p2p.empty()) return VMOE_ERR_NOT_READY;
  *bytes = p2p_chunk_stride(h) * h->p2p.size();
  return VMOE_OK;
}

namespace {
// One chunk of the fused forward on stream s (the whole pipeline of ep_p2p.cu).
int p2p_chunk(vmoe_handle* h, int c, const void* x, int64_t T, void* out, float* logits,
              char* ws, const P2PPlan& p, cudaStream_t s, bool prof) {
  const int64_t E = h->E, K = h->K, H = h->H;
  P2PChannel& ch = h->p2p[c];
  int32_t* idx = reinterpret_cast<int32_t*>(ws + p.idx);
  float* tw = reinterpret_cast<float*>(ws + p.w);
  int* hist = reinterpret_cast<int*>(ws + p.hist);
  float* psum = reinterpret_cast<float*>(ws + p.psum);
  int* excl = reinterpret_cast<int*>(ws + p.excl);
  int* counts = reinterpret_cast<int*>(ws + p.counts);
  float* psum_tot = reinterpret_cast<float*>(ws + p.psum_tot);
  int* offs = reinterpret_cast<int*>(ws + p.offs);
  float* aux = reinterpret_cast<float*>(ws + p.aux);
  const int nblk = static_cast<int>((T + kTileM - 1) / kTileM);

  P2PArgs a{};
  a.peer_base = ch.peers_dev;
  a.sig_off = h->p2p_sig_off;
  a.counts_off = h->p2p_counts_off;
  a.recv_off = h->p2p_recv_off;
  a.y_off = h->p2p_y_off;
  a.me = h->ep_rank;
  a.G = h->ep_size;
  a.E = static_cast<int>(E);
  a.El = static_cast<int>(h->E_local);
  a.K = static_cast<int>(K);
  a.H = H;
  a.cap_rows = h->p2p_cap_rows;
  a.row_align = static_cast<int>(h->tile_rows);
  a.epoch = ++ch.epoch;
  a.status = h->status;
  a.block_counter = ch.block_counter;
  a.dest_rank = reinterpret_cast<int32_t*>(ws + p.drank);
  a.dest_row = reinterpret_cast<int32_t*>(ws + p.drow);
  a.tile_expert = reinterpret_cast<int*>(ws + p.tiles);
  a.num_tiles = reinterpret_cast<int*>(ws + p.ntiles);
  a.push = h->p2p_push;
  a.ret_off = h->p2p_ret_off;
  a.back_off = h->p2p_back_off;
  a.back_rows = h->p2p_back_rows;
  a.peer_base_local = ch.region;

  cudaEvent_t* ev = prof ? &h->prof_ev[static_cast<size_t>(h->prof_count) * (kStages + 1)] : nullptr;
  int stage = 0;
  auto mark = [&]() {
    if (prof) cudaEventRecord(ev[stage], s);
    ++stage;
  };
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  int rc;
  mark();  // router
  if (T > 0 && (rc = run_router(h, x, T, logits, idx, tw, hist, psum, nullptr, s)) != VMOE_OK)
    return rc;
  mark();  // scan
  if ((rc = check(launch_scan_blocks(hist, psum, nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s), "scan")) != VMOE_OK)
    return rc;
  mark();  // plan (this chunk's counts) + publish counts to every rank
  if ((rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K), 0, 1,
                              offs, nullptr, nullptr, aux, nullptr, s), "plan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_p2p_publish(a, counts, s), "publish")) != VMOE_OK) return rc;
  // The chunks' dispatches run one after another (they share the links) and so do their
  // GEMMs (each fills every SM): chunk c's GEMMs can start as soon as its own rows arrived,
  // while chunk c+1's rows are still in flight and chunk c-1's outputs are combined.
  cudaError_t e;
  const bool chained = h->p2p.size() > 1;
  if (c > 0 && (e = cudaStreamWaitEvent(s, h->p2p_sent[c - 1], 0)) != cudaSuccess)
    return cuda_fail(h, e, "dispatch order");
  mark();  // dispatch over NVLink + wait for every rank's rows
  // with reserved SMs the transfer kernels claim 48 KB of shared memory per block, more
  // than a GEMM CTA leaves free, so they only run on the reserved SMs
  const size_t xfer_smem = h->p2p_reserve_sms > 0 ? 48 * 1024 : 0;
  const int gemm_sms = h->num_sms - h->p2p_reserve_sms;
  if ((rc = check(launch_p2p_dispatch(h->dtype, a, x, idx, excl, T, xfer_smem, s), "dispatch")) !=
      VMOE_OK)
    return rc;
  if (chained && (e = cudaEventRecord(h->p2p_sent[c], s)) != cudaSuccess)
    return cuda_fail(h, e, "dispatch order");
  if ((rc = check(launch_p2p_wait(a, 1, s), "wait rows")) != VMOE_OK) return rc;
  if (c > 0 && (e = cudaStreamWaitEvent(s, h->p2p_gemm_done[c - 1], 0)) != cudaSuccess)
    return cuda_fail(h, e, "gemm order");
  mark();  // gemm1 (inside run_expert_gemms: gemm1, mark, gemm2)
  if ((rc = run_expert_gemms(h, ch.region + h->p2p_recv_off, h->p2p_cap_rows, a.tile_expert,
                             a.num_tiles, ws + p.hbuf,
                             a.push ? nullptr : ch.region + h->p2p_y_off, H, s, mark, check,
                             gemm_sms, nullptr, a.push ? &a : nullptr)) != VMOE_OK)
    return rc;
  if (chained && (e = cudaEventRecord(h->p2p_gemm_done[c], s)) != cudaSuccess)
    return cuda_fail(h, e, "gemm order");
  mark();  // signal outputs ready, wait for every rank's, combine over NVLink
  if ((rc = check(launch_p2p_signal(a, 2, s), "signal outputs")) != VMOE_OK) return rc;
  if ((rc = check(launch_p2p_wait(a, 2, s), "wait outputs")) != VMOE_OK) return rc;
  if ((rc = check(a.push ? launch_p2p_combine_local(h->dtype, a, idx, tw, T, out, xfer_smem, s)
                         : launch_p2p_combine(h->dtype, a, idx, tw, T, out, xfer_smem, s),
                  "combine")) != VMOE_OK)
    return rc;
  mark();
  return VMOE_OK;
}
}  // namespace

int vmoe_ep_p2p_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                        float* router_logits, float* aux_loss, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (!h->p2p_connected) return fail(h, VMOE_ERR_NOT_READY, "vmoe_ep_p2p_connect has not been called");
  const int64_t E = h->E, K = h->K, H = h->H, T = tokens;
  if (T < 0 || T > h->p2p_max_tokens)
    return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be in [0, %lld] (got %lld)",
                static_cast<long long>(h->p2p_max_tokens), static_cast<long long>(T));
  if (T > 0 && (!x || !out)) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const int C = static_cast<int>(h->p2p.size());
  const size_t stride = p2p_chunk_stride(h);
  if (!workspace || workspace_bytes < stride * C)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", stride * C,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const P2PPlan p = make_p2p_plan(h, h->p2p_chunk_tokens);
  const size_t elt = dtype_bytes(h->dtype);
  const bool prof = h->prof_count < h->prof_slots;
  cudaError_t e;
  int rc;
  if (C == 1) {
    if ((rc = p2p_chunk(h, 0, x, T, out, router_logits, ws, p, s, prof)) != VMOE_OK) return rc;
  } else {
    // chunk c on its own stream: its dispatch and combine overlap the other chunks' GEMMs
    if ((e = cudaEventRecord(h->p2p_start, s)) != cudaSuccess) return cuda_fail(h, e, "event");
    for (int c = 0; c < C; ++c) {
      cudaStream_t sc = h->p2p_streams[c];
      if ((e = cudaStreamWaitEvent(sc, h->p2p_start, 0)) != cudaSuccess) return cuda_fail(h, e, "wait");
      const int64_t t0 = c * h->p2p_chunk_tokens;
      int64_t tc = T - t0;
      tc = tc < 0 ? 0 : (tc > h->p2p_chunk_tokens ? h->p2p_chunk_tokens : tc);
      const char* xc = static_cast<const char*>(x) + (tc > 0 ? t0 * H * elt : 0);
      char* oc = static_cast<char*>(out) + (tc > 0 ? t0 * H * elt : 0);
      float* lc = router_logits && tc > 0 ? router_logits + t0 * E : nullptr;
      if ((rc = p2p_chunk(h, c, tc > 0 ? xc : nullptr, tc, tc > 0 ? oc : nullptr, lc,
                          ws + c * stride, p, sc, prof && c == 0)) != VMOE_OK)
        return rc;
      if ((e = cudaEventRecord(h->p2p_done[c], sc)) != cudaSuccess) return cuda_fail(h, e, "event");
    }
    for (int c = 0; c < C; ++c)
      if ((e = cudaStreamWaitEvent(s, h->p2p_done[c], 0)) != cudaSuccess) return cuda_fail(h, e, "wait");
  }
  if (aux_loss) {  // the loss of the whole batch from every chunk's counts and sums
    if ((e = launch_aux_merge_ws(ws, stride, p.counts, p.psum_tot, C, T, static_cast<int>(E),
                                 static_cast<int>(K), aux_loss, s)) != cudaSuccess)
      return cuda_fail(h, e, "aux merge");
    ++h->last_launches;
  }
  if (prof) ++h->prof_count;
  return VMOE_OK;
}

int vmoe_ffn_create(const vmoe_config* cfg, int device, vmoe_handle** out) {
  if (!cfg || !out) return VMOE_ERR_INVALID_ARG;
  vmoe_config c = *cfg;
  c.num_experts = 2;  // passes the MoE checks; the handle below holds one expert
  c.top_k = 1;
  c.capacity = 0;
  const int rc = vmoe_create(&c, device, out);
  if (rc != VMOE_OK) return rc;
  vmoe_handle* h = *out;
  h->cfg.num_experts = 1;
  h->E = h->E_local = 1;
  h->K = 1;
  h->dense = true;
  return VMOE_OK;
}

namespace {
struct FfnPlan {
  int64_t max_rows = 0;
  size_t xp = 0, h = 0, y = 0, tiles = 0, ntiles = 0, total = 0;
};
FfnPlan make_ffn_plan(const vmoe_handle* h, int64_t T) {
  FfnPlan p;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const size_t elt = dtype_bytes(h->dtype);
  p.max_rows = round_up(T > 0 ? T : 1, h->tile_rows);
  p.xp = take(static_cast<size_t>(p.max_rows) * h->H * elt);
  p.h = take(static_cast<size_t>(p.max_rows) * h->Ipad * elt);
  p.y = take(static_cast<size_t>(p.max_rows) * h->Hpad * elt);
  p.tiles = take(p.max_rows / h->tile_rows * 4);
  p.ntiles = take(4);
  p.total = off;
  return p;
}
}  // namespace

int vmoe_ffn_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* bytes) {
  if (!h || !bytes || tokens < 0 || !h->dense) return VMOE_ERR_INVALID_ARG;
  *bytes = make_ffn_plan(h, tokens).total;
  return VMOE_OK;
}

int vmoe_ffn_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  if (!h->dense) return fail(h, VMOE_ERR_INVALID_ARG, "not a dense FFN handle (vmoe_ffn_create)");
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  const int64_t T = tokens, H = h->H;
  if (T < 0 || T >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_INVALID_ARG, "bad token count %lld", static_cast<long long>(T));
  if (T == 0) return VMOE_OK;
  if (!x || !out) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  const FfnPlan p = make_ffn_plan(h, T);
  if (!workspace || workspace_bytes < p.total)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", p.total,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const size_t elt = dtype_bytes(h->dtype);
  int* tiles = reinterpret_cast<int*>(ws + p.tiles);
  int* ntiles = reinterpret_cast<int*>(ws + p.ntiles);
  auto mark = []() {};
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  int rc;
  if ((rc = check(launch_fill_tiles(tiles, static_cast<int>(p.max_rows / h->tile_rows), ntiles, s),
                  "tile map")) != VMOE_OK)
    return rc;
  if (h->dtype == kBF16 && h->Hpad == H &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0) {
    // the tensor-core GEMMs read x and write out in place: the gate|up GEMM's A tensor map
    // holds T rows (the TMA zero-fills the rest of the last tile) and the down GEMM stores
    // only rows < T
    return run_expert_gemms(h, const_cast<void*>(x), p.max_rows, tiles, ntiles, ws + p.h, out, H,
                            s, mark, check, 0, nullptr, nullptr, T, T);
  }
  // x into a buffer padded to whole GEMM tiles (the GEMMs read full tiles)
  cudaError_t e = cudaMemcpyAsync(ws + p.xp, x, T * H * elt, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "x copy");
  if ((rc = run_expert_gemms(h, ws + p.xp, p.max_rows, tiles, ntiles, ws + p.h, ws + p.y, h->Hpad,
                             s, mark, check)) != VMOE_OK)
    return rc;
  e = cudaMemcpy2DAsync(out, H * elt, ws + p.y, h->Hpad * elt, H * elt, T,
                        cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "out copy");
  return VMOE_OK;
}

// ---- training: forward that keeps what the backward needs, and the backward -------------
namespace {

// The saved workspace of vmoe_forward_train: the forward's own plan (routing, slots, x_perm,
// h, y) plus the gate|up pre-activations and the router logits.
struct TrainPlan {
  Plan p;
  size_t gu = 0, logits = 0, total = 0;
};

TrainPlan make_train_plan(const vmoe_handle* h, int64_t T) {
  TrainPlan tp;
  tp.p = make_plan(h, T);
  size_t off = tp.p.total;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  tp.gu = take(static_cast<size_t>(tp.p.max_rows) * 2 * h->Ipad * 2);
  tp.logits = take(static_cast<size_t>(T) * h->E * 4);
  tp.total = off;
  return tp;
}

// Scratch of vmoe_backward.
struct BwdPlan {
  int64_t Tpad = 0;  // tokens padded to 128
  size_t dy, dgu, dxr, dw, dl, dl_bf, dxrt, dl_bs, total;
};

BwdPlan make_bwd_plan(const vmoe_handle* h, int64_t T, const Plan& p) {
  BwdPlan b{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const size_t R = static_cast<size_t>(p.max_rows);
  const size_t Hp = h->Hpad, Ip = h->Ipad;
  b.Tpad = round_up(T > 0 ? T : 1, kTileM);
  b.dy = take(R * Hp * 2);
  b.dgu = take(R * 2 * Ip * 2);
  b.dxr = take(R * Hp * 2);
  b.dw = take(static_cast<size_t>(T) * h->K * 4);
  b.dl = take(static_cast<size_t>(T) * h->E * 4);
  b.dl_bf = take(static_cast<size_t>(b.Tpad) * h->Epad64 * 2);
  b.dxrt = take(static_cast<size_t>(b.Tpad) * Hp * 2);
  b.dl_bs = take(static_cast<size_t>((T + 127) / 128) * h->E * 4);
  b.total = off;
  return b;
}

int check_trainable(vmoe_handle* h) {
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (!h->training) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_training has not been called");
  return VMOE_OK;
}

}  // namespace

int vmoe_set_training(vmoe_handle* h, int enable, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  if (!enable) {
    h->training = false;
    return VMOE_OK;
  }
  if (h->dtype != kBF16 || h->dense || h->ep_size > 1 || h->tile_rows != 2 * kTileM)
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE,
                "the backward runs on single-GPU bf16 MoE handles with the CTA-pair GEMMs");
  if (h->K > 32 || h->H % 8)
    return fail(h, VMOE_ERR_UNSUPPORTED_SHAPE, "the backward needs top_k <= 32 and hidden %% 8 == 0");
  DeviceGuard g(h->device);
  h->training = true;
  return h->ready ? make_training_copies(h, static_cast<cudaStream_t>(stream)) : VMOE_OK;
}

int vmoe_train_workspace_size(const vmoe_handle* h, int64_t tokens, size_t* saved_bytes,
                              size_t* scratch_bytes) {
  if (!h || tokens < 0 || !saved_bytes || !scratch_bytes) return VMOE_ERR_INVALID_ARG;
  const TrainPlan tp = make_train_plan(h, tokens);
  *saved_bytes = tp.total;
  *scratch_bytes = make_bwd_plan(h, tokens, tp.p).total;
  return VMOE_OK;
}

int vmoe_forward_train(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                       float* router_logits, float* aux_loss, void* saved, size_t saved_bytes,
                       void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  int rc = check_trainable(h);
  if (rc != VMOE_OK) return rc;
  const int64_t E = h->E, K = h->K, H = h->H, T = tokens;
  if (T < 1 || T * K + E * kTileM >= (static_cast<int64_t>(1) << 31))
    return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be in [1, 2^31 / top_k) (got %lld)",
                static_cast<long long>(T));
  if (!x || !out) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const TrainPlan tp = make_train_plan(h, T);
  if (!saved || saved_bytes < tp.total || (reinterpret_cast<uintptr_t>(saved) & 255u))
    return fail(h, VMOE_ERR_WORKSPACE, "saved workspace needs %zu bytes, 256-byte aligned",
                tp.total);
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(saved);
  const Plan& p = tp.p;
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  auto mark = []() {};
  int32_t* idx = reinterpret_cast<int32_t*>(ws + p.idx);
  float* tw = reinterpret_cast<float*>(ws + p.w);
  int* hist = reinterpret_cast<int*>(ws + p.hist);
  float* psum = reinterpret_cast<float*>(ws + p.psum);
  int* excl = reinterpret_cast<int*>(ws + p.excl);
  int* counts = reinterpret_cast<int*>(ws + p.counts);
  float* psum_tot = reinterpret_cast<float*>(ws + p.psum_tot);
  int* offs = reinterpret_cast<int*>(ws + p.offs);
  int* tiles = reinterpret_cast<int*>(ws + p.tiles);
  int* ntiles = reinterpret_cast<int*>(ws + p.ntiles);
  float* aux = aux_loss ? aux_loss : reinterpret_cast<float*>(ws + p.aux);
  int* slot = reinterpret_cast<int*>(ws + p.slot);
  float* logits = reinterpret_cast<float*>(ws + tp.logits);
  if ((rc = run_router(h, x, T, logits, idx, tw, hist, psum, nullptr, s)) != VMOE_OK) return rc;
  if ((rc = check(launch_scan_blocks(hist, psum, p.nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s), "scan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K),
                              h->cfg.capacity, static_cast<int>(h->tile_rows), offs, tiles, ntiles,
                              aux, nullptr, s), "plan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_dispatch(h->dtype, x, idx, excl, offs, T, static_cast<int>(H),
                                  static_cast<int>(E), static_cast<int>(K), h->cfg.capacity, slot,
                                  ws + p.xp, H, h->status, nullptr, s), "dispatch")) != VMOE_OK)
    return rc;
  // zero the padding rows of every segment: the weight gradients reduce over whole segments
  if ((rc = check(launch_zero_pad_rows(ws + p.xp, H * 2, H * 2, offs, counts, static_cast<int>(E),
                                       h->cfg.capacity, s), "pad rows")) != VMOE_OK)
    return rc;
  if ((rc = run_expert_gemms(h, ws + p.xp, p.max_rows, tiles, ntiles, ws + p.h, ws + p.y, h->Hpad,
                             s, mark, check, 0, ws + tp.gu)) != VMOE_OK)
    return rc;
  if ((rc = check(launch_combine(h->dtype, ws + p.y, h->Hpad, idx, tw, slot, T, static_cast<int>(H),
                                 static_cast<int>(K), out, nullptr, s), "combine")) != VMOE_OK)
    return rc;
  if (router_logits) {
    cudaError_t e = cudaMemcpyAsync(router_logits, logits, T * E * 4, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "logits copy");
  }
  return VMOE_OK;
}

int vmoe_backward(vmoe_handle* h, const void* x, const void* dout, int64_t tokens, const float* daux,
                  void* dx, const vmoe_grads* grads, const void* saved, size_t saved_bytes,
                  void* scratch, size_t scratch_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  h->last_launches = 0;
  int rc = check_trainable(h);
  if (rc != VMOE_OK) return rc;
  const int64_t E = h->E, K = h->K, H = h->H, I = h->I, T = tokens;
  const int64_t Hp = h->Hpad, Ip = h->Ipad;
  if (T < 1) return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be >= 1");
  if (!x || !dout || !dx || !grads || !grads->router_w || !grads->router_b || !grads->gate_w ||
      !grads->gate_b || !grads->up_w || !grads->up_b || !grads->down_w || !grads->down_b)
    return fail(h, VMOE_ERR_INVALID_ARG, "x, dout, dx and every gradient pointer are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dout) |
       reinterpret_cast<uintptr_t>(dx)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x, dout and dx must be 16-byte aligned");
  const TrainPlan tp = make_train_plan(h, T);
  const Plan& p = tp.p;
  const BwdPlan b = make_bwd_plan(h, T, p);
  if (!saved || saved_bytes < tp.total || (reinterpret_cast<uintptr_t>(saved) & 255u))
    return fail(h, VMOE_ERR_WORKSPACE, "saved workspace needs %zu bytes", tp.total);
  if (!scratch || scratch_bytes < b.total || (reinterpret_cast<uintptr_t>(scratch) & 255u))
    return fail(h, VMOE_ERR_WORKSPACE, "backward scratch needs %zu bytes, 256-byte aligned",
                b.total);
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const char* ws = static_cast<const char*>(saved);
  char* sc = static_cast<char*>(scratch);
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  const int32_t* idx = reinterpret_cast<const int32_t*>(ws + p.idx);
  const float* tw = reinterpret_cast<const float*>(ws + p.w);
  const int* counts = reinterpret_cast<const int*>(ws + p.counts);
  const int* offs = reinterpret_cast<const int*>(ws + p.offs);
  const int* tiles = reinterpret_cast<const int*>(ws + p.tiles);
  const int* ntiles = reinterpret_cast<const int*>(ws + p.ntiles);
  const int* slot = reinterpret_cast<const int*>(ws + p.slot);
  const float* logits = reinterpret_cast<const float*>(ws + tp.logits);
  const int64_t R = p.max_rows, max_tiles = R / h->tile_rows;
  cudaError_t e;
  const bool prof = h->bprof_count < h->prof_slots;
  cudaEvent_t* pev =
      prof ? &h->bprof_ev[static_cast<size_t>(h->bprof_count) * (kBwdStages + 1)] : nullptr;
  int stage = 0;
  auto mark = [&]() {
    if (prof) cudaEventRecord(pev[stage], s);
    ++stage;
  };

  // 1. combine backward: dy (expert-major rows) and dw; padding rows / columns zeroed
  mark();
  if (Hp != H && (e = cudaMemsetAsync(sc + b.dy, 0, R * Hp * 2, s)) != cudaSuccess)
    return cuda_fail(h, e, "dy clear");
  if ((rc = check(launch_combine_bwd(dout, ws + p.y, Hp, idx, tw, slot, T, static_cast<int>(H),
                                     static_cast<int>(K), sc + b.dy, Hp,
                                     reinterpret_cast<float*>(sc + b.dw), s), "combine bwd")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_zero_pad_rows(sc + b.dy, Hp * 2, Hp * 2, offs, counts, static_cast<int>(E),
                                       h->cfg.capacity, s), "dy pad rows")) != VMOE_OK)
    return rc;
  // 2. router backward
  mark();
  if ((rc = check(launch_router_bwd(logits, idx, reinterpret_cast<const float*>(sc + b.dw), counts,
                                    T, static_cast<int>(E), static_cast<int>(K), daux,
                                    reinterpret_cast<float*>(sc + b.dl), sc + b.dl_bf,
                                    static_cast<int>(h->Epad64),
                                    reinterpret_cast<float*>(sc + b.dl_bs), s), "router bwd")) != VMOE_OK)
    return rc;
  // 3. dh = dy W_d with the GLU / ERA backward epilogue -> dgu
  mark();
  char why[256];
  CUtensorMap m_dy, m_dgu, m_dl;
  if (!make_tmap_bf16(&m_dy, sc + b.dy, R, Hp, Hp, kTileM, why, sizeof(why)) ||
      !make_tmap_bf16(&m_dgu, sc + b.dgu, R, 2 * Ip, 2 * Ip, kTileM, why, sizeof(why)) ||
      !make_tmap_bf16(&m_dl, sc + b.dl_bf, b.Tpad, h->Epad64, h->Epad64, kTileM, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "backward tensor maps: %s", why);
  TcGemmArgs a1{};
  a1.num_m_tiles = ntiles;
  a1.tile_expert = tiles;
  a1.max_m_tiles = static_cast<int>(max_tiles);
  a1.num_experts = static_cast<int>(E);
  a1.n_tiles = static_cast<int>(h->Ipad2 / 256);
  a1.k_blocks = static_cast<int>(Hp / 64);
  a1.b_rows_per_expert = static_cast<int>(h->Ipad2);
  a1.out = sc + b.dgu;
  a1.ldo = 2 * Ip;
  a1.gamma = h->cfg.era_gamma;
  a1.status = h->status;
  a1.gu_in = ws + tp.gu;
  a1.gu_ld = 2 * Ip;
  a1.i_valid = Ip;
  if ((rc = check(launch_tc_gemm_pair_glu_bwd(m_dy, h->map_wdT, a1, max_tiles, h->num_sms, s),
                  "dh gemm")) != VMOE_OK)
    return rc;
  // 4. dx rows = dgu (gate|up)^T-major weights
  mark();
  TcGemmArgs a2{};
  a2.num_m_tiles = ntiles;
  a2.tile_expert = tiles;
  a2.max_m_tiles = static_cast<int>(max_tiles);
  a2.num_experts = static_cast<int>(E);
  a2.n_tiles = static_cast<int>(Hp / 256);
  a2.k_blocks = static_cast<int>(2 * Ip / 64);
  a2.b_rows_per_expert = static_cast<int>(Hp);
  a2.out = sc + b.dxr;
  a2.ldo = Hp;
  a2.bias = nullptr;
  a2.status = h->status;
  if ((rc = check(launch_tc_gemm_pair(false, m_dgu, h->map_guT, a2, max_tiles, h->num_sms, s),
                  "dx gemm")) != VMOE_OK)
    return rc;
  // 5. the router's share of dx: dlogits W_r
  mark();
  TcGemmArgs a3{};
  a3.num_m_tiles = nullptr;
  a3.m_tiles_host = static_cast<int>(b.Tpad / kTileM);
  a3.tile_expert = nullptr;
  a3.max_m_tiles = a3.m_tiles_host;
  a3.num_experts = 1;
  a3.n_tiles = static_cast<int>(Hp / 256);
  a3.k_blocks = static_cast<int>(h->Epad64 / 64);
  a3.b_rows_per_expert = 0;
  a3.out = sc + b.dxrt;
  a3.ldo = Hp;
  a3.bias = nullptr;
  a3.status = h->status;
  if ((rc = check(launch_tc_gemm(false, m_dl, h->map_wrT, a3, a3.m_tiles_host, h->num_sms, s),
                  "router dx gemm")) != VMOE_OK)
    return rc;
  // 6. dx = sum over each token's rows (ascending expert) + router share
  mark();
  if ((rc = check(launch_gather_dx(sc + b.dxr, Hp, sc + b.dxrt, Hp, idx, slot, T,
                                   static_cast<int>(H), static_cast<int>(K), dx, s), "dx gather")) != VMOE_OK)
    return rc;
  // 7. weight and bias gradients (fp32, straight into the caller's layout), operands read
  //    MN-major from their row-major activation buffers
  mark();
  CUtensorMap m_dyr, m_hr, m_dgur, m_xpr, m_xr, m_dlr;
  if (!make_tmap_bf16(&m_dyr, sc + b.dy, R, Hp, Hp, 64, why, sizeof(why)) ||
      !make_tmap_bf16(&m_hr, ws + p.h, R, Ip, Ip, 64, why, sizeof(why)) ||
      !make_tmap_bf16(&m_dgur, sc + b.dgu, R, 2 * Ip, 2 * Ip, 64, why, sizeof(why)) ||
      !make_tmap_bf16(&m_xpr, ws + p.xp, R, H, H, 64, why, sizeof(why)) ||
      !make_tmap_bf16(&m_xr, x, T, H, H, 64, why, sizeof(why)) ||
      !make_tmap_bf16(&m_dlr, sc + b.dl_bf, T, h->Epad64, h->Epad64, 64, why, sizeof(why)))
    return fail(h, VMOE_ERR_CUDA, "weight-gradient tensor maps: %s", why);
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  WgradArgs wd{};
  wd.seg_offs = offs;
  wd.rows_total = static_cast<int>(R);
  wd.num_experts = static_cast<int>(E);
  wd.m_tiles = static_cast<int>(Hp / kTileM);
  wd.n_tiles = static_cast<int>((Ip + 255) / 256);
  wd.m_valid = static_cast<int>(H);
  wd.n_valid = static_cast<int>(I);
  wd.out = grads->down_w;
  wd.ld_out = I;
  wd.out_expert_stride = H * I;
  wd.mode = 0;
  wd.vec_ok = (I % 4 == 0) && aligned(grads->down_w);
  wd.bias_out = grads->down_b;
  wd.status = h->status;
  // single-CTA weight gradients; VMOE_PAIR_WGRAD=1 selects the CTA-pair kernel (M tiles of
  // 256), which measured slower here: with both operands read MN-major the tensor pipe,
  // not the operand traffic the pair halves, is the limit
  const char* pw = getenv("VMOE_PAIR_WGRAD");
  const bool pair_wgrad = pw && pw[0] == '1';
  auto wgrad = [&](const CUtensorMap& a, const CUtensorMap& bm, WgradArgs wa) {
    if (pair_wgrad) {
      wa.m_tiles = (wa.m_tiles + 1) / 2;  // 128-row tiles -> 256-row pair tiles
      return launch_wgrad_pair(a, bm, wa, h->num_sms, s);
    }
    return launch_wgrad(a, bm, wa, h->num_sms, s);
  };
  if ((rc = check(wgrad(m_dyr, m_hr, wd), "dW_down")) != VMOE_OK) return rc;
  mark();
  WgradArgs wg = wd;
  wg.m_tiles = static_cast<int>(2 * Ip / kTileM);
  wg.n_tiles = static_cast<int>(Hp / 256);
  wg.m_valid = static_cast<int>(I);
  wg.n_valid = static_cast<int>(H);
  wg.out = grads->gate_w;
  wg.out2 = grads->up_w;
  wg.ld_out = H;
  wg.out_expert_stride = I * H;
  wg.mode = 1;
  wg.vec_ok = (H % 4 == 0) && aligned(grads->gate_w) && aligned(grads->up_w);
  wg.bias_out = grads->gate_b;
  wg.bias_out2 = grads->up_b;
  if ((rc = check(wgrad(m_dgur, m_xpr, wg), "dW_gate_up")) != VMOE_OK) return rc;
  mark();
  WgradArgs wr{};
  wr.seg_offs = nullptr;
  wr.seg_rows_host = static_cast<int>(b.Tpad);
  wr.rows_total = static_cast<int>(b.Tpad);
  wr.num_experts = 1;
  wr.m_tiles = static_cast<int>((h->Epad64 + kTileM - 1) / kTileM);
  wr.n_tiles = static_cast<int>(Hp / 256);
  wr.m_valid = static_cast<int>(E);
  wr.n_valid = static_cast<int>(H);
  wr.out = grads->router_w;
  wr.ld_out = H;
  wr.out_expert_stride = 0;
  wr.mode = 0;
  wr.vec_ok = (H % 4 == 0) && aligned(grads->router_w);
  wr.status = h->status;
  if ((rc = check(wgrad(m_dlr, m_xr, wr), "dW_router")) != VMOE_OK) return rc;
  // the router bias: per-block sums of dlogits, added in block order
  if ((rc = check(launch_segment_sum(reinterpret_cast<const float*>(sc + b.dl_bs), E, nullptr,
                                     static_cast<int>((T + 127) / 128), static_cast<int>(E), 128,
                                     grads->router_b, nullptr, static_cast<int>(E), false, s),
                  "db_router")) != VMOE_OK)
    return rc;
  mark();
  if (prof) ++h->bprof_count;
  return VMOE_OK;
}

int vmoe_device_status(vmoe_handle* h, int32_t* code, void* stream) {
  if (!h || !code) return VMOE_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, h->status, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(h->status, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(h, e, "status read");
  *code = v;
  if (v == 0) return VMOE_OK;
  if (v >= 0x101 && v <= 0x1FF)
    return fail(h, VMOE_ERR_TIMEOUT, "a bounded device wait gave up (status 0x%x)", v);
  return fail(h, VMOE_ERR_DEVICE_STATUS, "device status 0x%x", v);
}

int vmoe_set_profiling(vmoe_handle* h, int n) {
  if (!h || n < 0) return VMOE_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  for (cudaEvent_t ev : h->prof_ev) cudaEventDestroy(ev);
  for (cudaEvent_t ev : h->bprof_ev) cudaEventDestroy(ev);
  h->prof_ev.clear();
  h->bprof_ev.clear();
  h->prof_slots = 0;
  h->prof_count = 0;
  h->bprof_count = 0;
  if (n == 0) return VMOE_OK;
  h->prof_ev.resize(static_cast<size_t>(n) * (kStages + 1));
  h->bprof_ev.resize(static_cast<size_t>(n) * (kBwdStages + 1));
  for (auto* ring : {&h->prof_ev, &h->bprof_ev}) {
    for (auto& ev : *ring) {
      cudaError_t e = cudaEventCreate(&ev);
      if (e != cudaSuccess) {
        ev = nullptr;
        return cuda_fail(h, e, "profiling events");
      }
    }
  }
  h->prof_slots = n;
  return VMOE_OK;
}

int vmoe_backward_stage_times(vmoe_handle* h, float* ms, int n, int* n_out, int* calls) {
  if (!h || !ms || n < 0) return VMOE_ERR_INVALID_ARG;
  if (h->bprof_count == 0) return fail(h, VMOE_ERR_NOT_READY, "no profiled backward recorded");
  DeviceGuard g(h->device);
  const int m = n < kBwdStages ? n : kBwdStages;
  for (int i = 0; i < m; ++i) ms[i] = 0.f;
  for (int f = 0; f < h->bprof_count; ++f) {
    cudaEvent_t* ev = &h->bprof_ev[static_cast<size_t>(f) * (kBwdStages + 1)];
    cudaError_t e = cudaEventSynchronize(ev[kBwdStages]);
    if (e != cudaSuccess) return cuda_fail(h, e, "stage timing");
    for (int i = 0; i < m; ++i) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
      if (e != cudaSuccess) return cuda_fail(h, e, "stage timing");
      ms[i] += t;
    }
  }
  for (int i = 0; i < m; ++i) ms[i] /= static_cast<float>(h->bprof_count);
  if (n_out) *n_out = m;
  if (calls) *calls = h->bprof_count;
  h->bprof_count = 0;
  return VMOE_OK;
}

const char* vmoe_backward_stage_name(int stage) {
  return stage >= 0 && stage < kBwdStages ? kBwdStageNames[stage] : "";
}

int vmoe_stage_times(vmoe_handle* h, float* ms, int n, int* n_out, int* forwards) {
  if (!h || !ms || n < 0) return VMOE_ERR_INVALID_ARG;
  if (h->prof_count == 0) return fail(h, VMOE_ERR_NOT_READY, "no profiled forward recorded");
  DeviceGuard g(h->device);
  const int m = n < kStages ? n : kStages;
  for (int i = 0; i < m; ++i) ms[i] = 0.f;
  for (int f = 0; f < h->prof_count; ++f) {
    cudaEvent_t* ev = &h->prof_ev[static_cast<size_t>(f) * (kStages + 1)];
    cudaError_t e = cudaEventSynchronize(ev[kStages]);
    if (e != cudaSuccess) return cuda_fail(h, e, "stage timing");
    for (int i = 0; i < m; ++i) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
      if (e != cudaSuccess) return cuda_fail(h, e, "stage timing");
      ms[i] += t;
    }
  }
  for (int i = 0; i < m; ++i) ms[i] /= static_cast<float>(h->prof_count);
  if (n_out) *n_out = m;
  if (forwards) *forwards = h->prof_count;
  h->prof_count = 0;
  return VMOE_OK;
}

int vmoe_last_launch_count(const vmoe_handle* h) { return h ? h->last_launches : 0; }

int vmoe_gemm_tile_rows(const vmoe_handle* h) { return h ? h->tile_rows : 0; }

}  // extern "C"
