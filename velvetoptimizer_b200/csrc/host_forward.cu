// C-ABI forward on host buffers (vmoe_forward_host): the batch's copy-in, the chunks'
// forwards and the copy-out overlap on two internal copy streams; chunks carry their
// experts' partial GEMM tiles into the next chunk.
#include "moe_host.h"

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
    hp.fwd = take(make_plan(h, T).total);  // the whole batch in one forward_batch
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

}  // namespace

int vmoe_host::ensure_host_streams(vmoe_handle* h) {
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

extern "C" {

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

}  // extern "C"
