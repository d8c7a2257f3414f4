// C-ABI training: the forward that keeps what the backward needs (vmoe_forward_train) and
// the backward (vmoe_backward): dx and the fp32 gradients of the router and of every expert.
#include "moe_host.h"

extern "C" {

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
  // the inference forward's routing blocks (only the forward's scan reads their histograms),
  // so that routing, aux and outputs are bit-identical to vmoe_forward's
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
  if ((rc = run_router(h, x, T, logits, idx, tw, hist, psum, nullptr, s, p.rb)) != VMOE_OK)
    return rc;
  if ((rc = check(launch_scan_blocks(hist, psum, p.nblk, static_cast<int>(E), excl, counts,
                                     psum_tot, s), "scan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_plan(counts, psum_tot, T, static_cast<int>(E), static_cast<int>(K),
                              h->cfg.capacity, static_cast<int>(h->tile_rows), offs, tiles, ntiles,
                              aux, nullptr, s), "plan")) != VMOE_OK)
    return rc;
  if ((rc = check(launch_dispatch(h->dtype, x, idx, excl, offs, T, static_cast<int>(H),
                                  static_cast<int>(E), static_cast<int>(K), h->cfg.capacity, slot,
                                  ws + p.xp, H, h->status, nullptr, s, p.rb), "dispatch")) != VMOE_OK)
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
  NvtxStages nvtx(kNvtxBwdStageNames, kBwdStages);
  auto mark = [&]() {
    if (prof) cudaEventRecord(pev[stage], s);
    nvtx.next(stage);
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

}  // extern "C"
