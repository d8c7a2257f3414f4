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
#include "moe_host.h"

namespace vmoe_host {

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

Plan make_plan(const vmoe_handle* h, int64_t T, int rb) {
  Plan p;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const int64_t E = h->E, K = h->K;
  const size_t elt = dtype_bytes(h->dtype);
  p.rb = rb > 0 ? rb : routing_block(h, T);
  p.nblk = static_cast<int>((T + p.rb - 1) / p.rb);
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
  p.ready = take(E * 4);
  p.total = off;
  return p;
}

// Router + softmax + top-K + per-block histogram / probability sums: on the tensor cores
// for bf16 with E <= 64, on CUDA cores otherwise (fp32 parity, or wider routers).
// With `ln` the router reads LayerNorm(x) without materialising it: the tensor-core router
// through the folded weights (and its own row statistics), the CUDA-core router through a
// statistics pass and normalisation on load.
int run_router(vmoe_handle* h, const void* x, int64_t T, float* logits, int32_t* idx, float* tw,
               int* hist, float* psum, const LnArgs* ln, cudaStream_t s, int rb) {
  const int64_t H = h->H;
  cudaError_t e;
  if (h->dtype == kBF16 && h->router_bn > 0) {
    char why[256];
    CUtensorMap map_x;
    if (!make_tmap_bf16(&map_x, x, T, H, H, static_cast<uint32_t>(rb), why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "x tensor map: %s", why);
    TcGemmArgs a{};
    a.num_m_tiles = nullptr;
    a.route_rows = rb;
    a.m_tiles_host = static_cast<int>((T + rb - 1) / rb);
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
    if (rb != kTileM)
      return fail(h, VMOE_ERR_INVALID_ARG, "the CUDA-core router routes 128-token blocks");
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
                  bool prenorm) {
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
  int* ready = reinterpret_cast<int*>(ws + p.ready);
  void* xp = ws + p.xp;
  void* hb = ws + p.h;
  void* yb = ws + p.y;

  cudaEvent_t* ev = prof ? &h->prof_ev[static_cast<size_t>(h->prof_count) * (kStages + 1)] : nullptr;
  int stage = 0;
  NvtxStages nvtx(kNvtxStageNames, kStages);
  // a decode batch's kernels each fit in one wave: launch them with programmatic dependent
  // launch, each overlapping the end of the one before (VMOE_PDL=0 at handle creation: off)
  PdlScope pdl(use_decode_gemms(h, T) && h->decode_pdl);
  auto mark = [&]() {
    if (prof) cudaEventRecord(ev[stage], s);
    nvtx.next(stage);
    ++stage;
  };
  auto check = [&](cudaError_t err, const char* what) -> int {
    if (err != cudaSuccess) return cuda_fail(h, err, what);
    ++h->last_launches;
    return VMOE_OK;
  };
  int rc;
  // decode-sized batches: segments padded to 16 rows for the swapped-operand GEMMs, which
  // need no tile map, and the scan and plan run inside the dispatch (two launches fewer)
  const bool decode = use_decode_gemms(h, T);
  const bool fold_plan = decode && h->decode_fold_plan && p.nblk <= 32 && !psum_tot_out;
  mark();
  if ((rc = run_router(h, x, T, router_logits, idx, tw, hist, psum, ln, s, p.rb)) != VMOE_OK)
    return rc;
  mark();
  if (!fold_plan &&
      (rc = check(launch_scan_blocks(hist, psum, p.nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s),
                  "scan")) != VMOE_OK)
    return rc;
  mark();
  if (!fold_plan &&
      (rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K),
                              h->cfg.capacity, segment_align(h, T), offs,
                              decode ? nullptr : tiles, decode ? nullptr : ntiles, aux,
                              expert_counts, s, decode ? ready : nullptr),
                  "plan")) != VMOE_OK)
    return rc;
  mark();
  const DispatchPlan folded{hist, psum, segment_align(h, T), offs, expert_counts, aux, ready,
                            static_cast<int>(E)};
  if ((rc = check(launch_dispatch(h->dtype, x, idx, excl, offs, T, static_cast<int>(H),
                                  static_cast<int>(E), static_cast<int>(K), h->cfg.capacity, slot,
                                  xp, H, h->status, ln, s, p.rb, fold_plan ? &folded : nullptr),
                  "dispatch")) != VMOE_OK)
    return rc;
  mark();
  if ((rc = decode ? run_decode_gemms(h, xp, p.max_rows, offs, hb, yb, T, ready, s, mark, check)
                   : run_expert_gemms(h, xp, p.max_rows, tiles, ntiles, hb, yb, h->Hpad, s, mark,
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
    const int64_t E = h->E, H = h->H, Er = router_rows(h);
    int rc;
    if (!h->w_r_ln) {  // zero rows past E (see router_rows); the fold writes rows < E
      if ((rc = alloc(h, &h->w_r_ln, Er * H * 2, "folded router weight")) != VMOE_OK) return rc;
      const cudaError_t z = cudaMemsetAsync(h->w_r_ln, 0, Er * H * 2, s);
      if (z != cudaSuccess) return cuda_fail(h, z, "folded router weight");
    }
    if (!h->b_r_ln && (rc = alloc(h, &h->b_r_ln, E * 4, "folded router bias")) != VMOE_OK) return rc;
    if (!h->c_ln && (rc = alloc(h, &h->c_ln, E * 4, "folded router sums")) != VMOE_OK) return rc;
    cudaError_t e = launch_fold_router_ln(h->w_r, h->b_r, h->ln_w, h->ln_b, static_cast<int>(E),
                                          static_cast<int>(H), h->w_r_ln, h->b_r_ln, h->c_ln, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "router LayerNorm fold");
    char why[256];
    if (!make_tmap_bf16(&h->map_wr_ln, h->w_r_ln, Er, H, H, static_cast<uint32_t>(h->router_bn),
                        why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "folded router tensor map: %s", why);
  }
  h->ln_ready = true;
  return VMOE_OK;
}

}  // namespace vmoe_host

namespace {

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
    // forwards of at most this many tokens run the swapped-operand (decode) GEMMs;
    // VMOE_DECODE_MAX_TOKENS lowers it (0: never)
    h->decode_max_tokens = kDecodeMaxTokens;
    if (const char* f = getenv("VMOE_DECODE_FUSED")) h->decode_fused = f[0] != '0';
    if (const char* f = getenv("VMOE_PDL")) h->decode_pdl = f[0] != '0';
    if (const char* f = getenv("VMOE_FOLD_PLAN")) h->decode_fold_plan = f[0] != '0';
    if (const char* f = getenv("VMOE_GEMM1_BAND")) h->gemm1_band = static_cast<int>(strtol(f, nullptr, 10));
    if (const char* f = getenv("VMOE_GEMM2_BAND")) h->gemm2_band = static_cast<int>(strtol(f, nullptr, 10));
    if (const char* d = getenv("VMOE_DECODE_MAX_TOKENS")) {
      const long v = strtol(d, nullptr, 10);
      h->decode_max_tokens = v < 0 ? 0 : (v > kDecodeMaxTokens ? kDecodeMaxTokens : static_cast<int>(v));
    }
  } else {
    h->Ipad = h->I;
    h->Hpad = h->H;
  }
  DeviceGuard g(device);
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&h->l2_bytes, cudaDevAttrL2CacheSize, device);
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

int vmoe_set_weights(vmoe_handle* h, const vmoe_weights* w, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  if (!w) return fail(h, VMOE_ERR_INVALID_ARG, "weights is NULL");
  if ((!w->router_w && !h->dense) || !w->gate_w || !w->up_w || !w->down_w)
    return fail(h, VMOE_ERR_INVALID_ARG, "router_w, gate_w, up_w and down_w are required");
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The packed buffers are sized by the handle's config alone, so a repack (after every
  // optimizer step of a training loop) reuses them: the pack kernels are ordered after any
  // forward already enqueued on `s`, and no cudaFree synchronises the device.
  h->ready = false;
  h->ln_ready = false;
  const int64_t E = h->E, H = h->H, I = h->I, Ipad = h->Ipad, Hpad = h->Hpad;
  const int64_t El = h->E_local;  // experts held by this handle (E without expert parallelism)
  const size_t elt = dtype_bytes(h->dtype);
  const bool bf16 = h->dtype == kBF16;
  const int R = h->cfg.lora_rank;
  int rc;
  // the tensor-core router reads W_r in boxes of its N tile (16/32/64 rows): rows past E
  // are zero, so no box reaches outside the tensor
  const int64_t Er = router_rows(h);
  if ((rc = alloc_once(h, &h->w_r, Er * H * elt, "router weight")) != VMOE_OK) return rc;
  if ((rc = alloc_once(h, &h->b_r, E * 4, "router bias")) != VMOE_OK) return rc;
  const int64_t gu_rows = bf16 ? 2 * Ipad : I;
  if ((rc = alloc_once(h, &h->w_g, El * gu_rows * H * elt, "gate weight")) != VMOE_OK) return rc;
  if ((rc = alloc_once(h, &h->b_g, El * gu_rows * 4, "gate bias")) != VMOE_OK) return rc;
  if (!bf16) {
    if ((rc = alloc_once(h, &h->w_u, El * I * H * elt, "up weight")) != VMOE_OK) return rc;
    if ((rc = alloc_once(h, &h->b_u, El * I * 4, "up bias")) != VMOE_OK) return rc;
  }
  if ((rc = alloc_once(h, &h->w_d, El * Hpad * Ipad * elt, "down weight")) != VMOE_OK) return rc;
  if ((rc = alloc_once(h, &h->b_d, El * Hpad * 4, "down bias")) != VMOE_OK) return rc;

  cudaError_t e;
  // router: plain copy of W_r, bias to fp32 (zeros for a dense handle)
  if (w->router_w)
    e = cudaMemcpyAsync(h->w_r, w->router_w, E * H * elt, cudaMemcpyDeviceToDevice, s);
  else
    e = cudaMemsetAsync(h->w_r, 0, E * H * elt, s);
  if (e == cudaSuccess && Er > E)
    e = cudaMemsetAsync(static_cast<char*>(h->w_r) + E * H * elt, 0, (Er - E) * H * elt, s);
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
        !make_tmap_bf16(&h->map_wr, h->w_r, Er, H, H, static_cast<uint32_t>(h->router_bn), why,
                        sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "router tensor map: %s", why);
    // B tiles: 256 rows per CTA, or 128 per CTA of a pair
    const uint32_t b_box = h->tile_rows == kTileM ? 256u : 128u;
    if (!make_tmap_bf16(&h->map_wgu, h->w_g, El * 2 * Ipad, H, H, b_box, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "gate/up tensor map: %s", why);
    if (!make_tmap_bf16(&h->map_wd, h->w_d, El * Hpad, Ipad, Ipad, b_box, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "down tensor map: %s", why);
    if (!make_tmap_bf16(&h->map_wgu_dec, h->w_g, El * 2 * Ipad, H, H, 64, why, sizeof(why)) ||
        !make_tmap_bf16(&h->map_wd_dec, h->w_d, El * Hpad, Ipad, Ipad, 128, why, sizeof(why)))
      return fail(h, VMOE_ERR_CUDA, "decode weight tensor maps: %s", why);
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
  const int64_t E = h->E, K = h->K, T = tokens;
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

int vmoe_segment_align(const vmoe_handle* h, int64_t tokens) {
  return h && tokens >= 0 ? segment_align(h, tokens) : 0;
}

}  // extern "C"
