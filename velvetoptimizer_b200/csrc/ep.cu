// C-ABI expert parallelism: the staged transport (route / NCCL all-to-all-v by the caller /
// experts / combine) and the fused NVLink transport (peer-memory dispatch and combine inside
// the forward, token chunks on internal streams).
#include "moe_host.h"

namespace {

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

}  // namespace

extern "C" {

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
  // with token chunks, 16 SMs stay out of the chunked GEMM grid for the NVLink transfer
  // kernels of the other chunks (measured on 4 GPUs, 4 chunks: 14.7 ms per step with none
  // reserved, 13.8 with 8, 13.5 with 16); VMOE_EP_RESERVE_SMS=n overrides
  h->p2p_reserve_sms = chunks > 1 ? 16 : 0;
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
  NvtxStages nvtx(kNvtxStageNames, kStages);
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
  if ((rc = check(launch_p2p_dispatch(h->dtype, a, x, idx, excl, T, xfer_smem, !chained, s),
                  "dispatch")) != VMOE_OK)
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

namespace {
// Host buffers of vmoe_ep_p2p_forward_host: each chunk's rows are copied in on h->host_in
// before the chunk starts and copied out on h->host_out after it ends.
struct HostIO {
  const char* x_host;
  char* out_host;
  char* x_dev;    // staging, >= tokens rows
  char* out_dev;  // staging, >= tokens rows
};

// One fused expert-parallel forward (every rank calls it): on `s` with one chunk and no host
// buffers, else chunk c on internal stream c (its NVLink exchange overlapping the other
// chunks' GEMMs, and with host buffers its copies overlapping the other chunks too).
int ep_p2p_run(vmoe_handle* h, const void* x, int64_t T, void* out, float* router_logits,
               float* aux_loss, char* ws, cudaStream_t s, const HostIO* io) {
  const int64_t E = h->E, K = h->K, H = h->H;
  const int C = static_cast<int>(h->p2p.size());
  const size_t stride = p2p_chunk_stride(h);
  const P2PPlan p = make_p2p_plan(h, h->p2p_chunk_tokens);
  const size_t row = static_cast<size_t>(H) * dtype_bytes(h->dtype);
  const bool prof = h->prof_count < h->prof_slots;
  cudaError_t e;
  int rc;
  if (C == 1 && !io) {
    if ((rc = p2p_chunk(h, 0, x, T, out, router_logits, ws, p, s, prof)) != VMOE_OK) return rc;
  } else {
    if ((e = cudaEventRecord(h->p2p_start, s)) != cudaSuccess) return cuda_fail(h, e, "event");
    if (io) {  // the copy-in may overwrite the staging rows only after earlier work on s
      if ((e = cudaStreamWaitEvent(h->host_in, h->p2p_start, 0)) != cudaSuccess)
        return cuda_fail(h, e, "wait");
      if ((e = cudaStreamWaitEvent(h->host_out, h->p2p_start, 0)) != cudaSuccess)
        return cuda_fail(h, e, "wait");
    }
    for (int c = 0; c < C; ++c) {
      cudaStream_t sc = h->p2p_streams[c];
      if ((e = cudaStreamWaitEvent(sc, h->p2p_start, 0)) != cudaSuccess) return cuda_fail(h, e, "wait");
      const int64_t t0 = c * h->p2p_chunk_tokens;
      int64_t tc = T - t0;
      tc = tc < 0 ? 0 : (tc > h->p2p_chunk_tokens ? h->p2p_chunk_tokens : tc);
      const char* xbase = io ? io->x_dev : static_cast<const char*>(x);
      char* obase = io ? io->out_dev : static_cast<char*>(out);
      if (io) {
        if (tc > 0 && (e = cudaMemcpyAsync(io->x_dev + t0 * row, io->x_host + t0 * row, tc * row,
                                           cudaMemcpyHostToDevice, h->host_in)) != cudaSuccess)
          return cuda_fail(h, e, "copy in");
        if ((e = cudaEventRecord(h->host_in_ev[c], h->host_in)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(sc, h->host_in_ev[c], 0)) != cudaSuccess)
          return cuda_fail(h, e, "copy-in order");
      }
      const char* xc = tc > 0 ? xbase + t0 * row : nullptr;
      char* oc = tc > 0 ? obase + t0 * row : nullptr;
      float* lc = router_logits && tc > 0 ? router_logits + t0 * E : nullptr;
      if ((rc = p2p_chunk(h, c, xc, tc, oc, lc, ws + c * stride, p, sc, prof && c == 0)) != VMOE_OK)
        return rc;
      if ((e = cudaEventRecord(h->p2p_done[c], sc)) != cudaSuccess) return cuda_fail(h, e, "event");
      if (io) {
        if ((e = cudaStreamWaitEvent(h->host_out, h->p2p_done[c], 0)) != cudaSuccess)
          return cuda_fail(h, e, "copy-out order");
        if (tc > 0 && (e = cudaMemcpyAsync(io->out_host + t0 * row, io->out_dev + t0 * row,
                                           tc * row, cudaMemcpyDeviceToHost, h->host_out)) !=
                          cudaSuccess)
          return cuda_fail(h, e, "copy out");
      }
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
  if (io) {  // s ends after the last copy-out
    if ((e = cudaEventRecord(h->host_out_done, h->host_out)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(s, h->host_out_done, 0)) != cudaSuccess)
      return cuda_fail(h, e, "copy-out join");
  }
  if (prof) ++h->prof_count;
  return VMOE_OK;
}

int check_p2p_call(vmoe_handle* h, int64_t T) {
  h->last_launches = 0;
  if (!h->ready) return fail(h, VMOE_ERR_NOT_READY, "vmoe_set_weights has not been called");
  if (!h->p2p_connected) return fail(h, VMOE_ERR_NOT_READY, "vmoe_ep_p2p_connect has not been called");
  if (T < 0 || T > h->p2p_max_tokens)
    return fail(h, VMOE_ERR_INVALID_ARG, "tokens must be in [0, %lld] (got %lld)",
                static_cast<long long>(h->p2p_max_tokens), static_cast<long long>(T));
  return VMOE_OK;
}

void CUDART_CB write_nan_host(void* p) { *static_cast<float*>(p) = __builtin_nanf(""); }
}  // namespace

int vmoe_ep_p2p_forward(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                        float* router_logits, float* aux_loss, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  const int64_t T = tokens;
  int rc = check_p2p_call(h, T);
  if (rc != VMOE_OK) return rc;
  if (T > 0 && (!x || !out)) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(h, VMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const size_t need = p2p_chunk_stride(h) * h->p2p.size();
  if (!workspace || workspace_bytes < need)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", need,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceGuard g(h->device);
  return ep_p2p_run(h, x, T, out, router_logits, aux_loss, static_cast<char*>(workspace),
                    static_cast<cudaStream_t>(stream), nullptr);
}

int vmoe_ep_p2p_host_workspace_size(const vmoe_handle* h, size_t* bytes) {
  if (!h || !bytes) return VMOE_ERR_INVALID_ARG;
  if (h->p2p.empty()) return VMOE_ERR_NOT_READY;
  const size_t rows = round_up(h->p2p_max_tokens > 0 ? h->p2p_max_tokens : 1, 16) *
                      static_cast<size_t>(h->H) * dtype_bytes(h->dtype);
  *bytes = p2p_chunk_stride(h) * h->p2p.size() + 2 * round_up(rows, 256) + 256;
  return VMOE_OK;
}

int vmoe_ep_p2p_forward_host(vmoe_handle* h, const void* x_host, int64_t tokens, void* out_host,
                             float* aux_loss_host, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  const int64_t T = tokens;
  int rc = check_p2p_call(h, T);
  if (rc != VMOE_OK) return rc;
  if (T > 0 && (!x_host || !out_host)) return fail(h, VMOE_ERR_INVALID_ARG, "x and out are required");
  size_t need = 0;
  vmoe_ep_p2p_host_workspace_size(h, &need);
  if (!workspace || workspace_bytes < need)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", need,
                workspace ? workspace_bytes : static_cast<size_t>(0));
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(h, VMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceGuard g(h->device);
  if ((rc = ensure_host_streams(h)) != VMOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const size_t rows = round_up(h->p2p_max_tokens > 0 ? h->p2p_max_tokens : 1, 16) *
                      static_cast<size_t>(h->H) * dtype_bytes(h->dtype);
  const size_t x_off = p2p_chunk_stride(h) * h->p2p.size();
  const size_t out_off = x_off + round_up(rows, 256), aux_off = out_off + round_up(rows, 256);
  HostIO io{static_cast<const char*>(x_host), static_cast<char*>(out_host), ws + x_off,
            ws + out_off};
  float* aux_dev = reinterpret_cast<float*>(ws + aux_off);
  rc = ep_p2p_run(h, nullptr, T, nullptr, nullptr, aux_loss_host ? aux_dev : nullptr, ws, s, &io);
  if (rc != VMOE_OK) return rc;
  if (aux_loss_host) {
    cudaError_t e = T > 0 ? cudaMemcpyAsync(aux_loss_host, aux_dev, 4, cudaMemcpyDeviceToHost, s)
                          : cudaLaunchHostFunc(s, write_nan_host, aux_loss_host);
    if (e != cudaSuccess) return cuda_fail(h, e, "aux copy");
  }
  return VMOE_OK;
}

}  // extern "C"
