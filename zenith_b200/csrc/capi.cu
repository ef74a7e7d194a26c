// extern "C" entry points of libzenith_ssd.so (declared in include/zb_ssd.h): argument
// validation, workspace planning and dispatch to the kernel families.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "ssd_kernels.h"
#include "ssd_tc.h"

using namespace zb;

namespace zb {
static std::atomic<uint64_t> g_launches{0};
void note_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device) and size: later calls
// with a size already granted make no CUDA call, so launches can also be captured in CUDA graphs.
int dyn_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> granted;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ZB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  int& have = granted[{fn, dev}];
  if (bytes <= have) return ZB_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return ZB_ERR_CUDA;
  have = bytes;
  return ZB_OK;
}
}  // namespace zb

namespace {

thread_local char g_cuda_err[256] = "";

int cuda_fail(cudaError_t e) {
  snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return ZB_ERR_CUDA;
}

size_t dtype_size(int dt) {
  switch (dt) {
    case ZB_F32: return 4;
    case ZB_BF16: return 2;
    case ZB_F16: return 2;
    case ZB_F64: return 8;
    default: return 0;
  }
}

enum Kind { kSimt = 0, kTc = 1 };

struct Plan {
  Kind kind;
  int L, nc;
  size_t acc;           // bytes of one state element
  size_t states_bytes;  // saved chunk states
  size_t sync_bytes;    // ticket + flags
  size_t gchain_bytes;  // backward gradient chain
  size_t grp_bytes;     // per-head q/k/kp gradients when G < H
  size_t tc_fwd_ws, tc_bwd_ws;
};

bool view_ok(const zb_view& v, size_t esz) {
  return v.ptr != nullptr && (reinterpret_cast<uintptr_t>(v.ptr) % esz) == 0;
}

int validate(const zb_ssd_args* a, bool backward) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0 || a->chunk_size <= 0)
    return ZB_ERR_SHAPE;
  if (a->T % a->chunk_size != 0) return ZB_ERR_SHAPE;  // mamba3.py:33
  if (a->H % a->G != 0) return ZB_ERR_SHAPE;
  // work units are numbered in 32 bits on the device
  if ((double)a->B * (double)a->H * (double)a->T > 2147483647.0) return ZB_ERR_SHAPE;
  const size_t e = dtype_size(a->dtype), es = dtype_size(a->scalar_dtype);
  if (!e || !es) return ZB_ERR_DTYPE;
  if ((a->dtype == ZB_F64) != (a->scalar_dtype == ZB_F64)) return ZB_ERR_DTYPE;
  const zb_view* vec[] = {&a->x, &a->q, &a->k, &a->kp, &a->xp};
  for (auto v : vec)
    if (!view_ok(*v, e)) return ZB_ERR_LAYOUT;
  const zb_view* sc[] = {&a->adt, &a->gamma, &a->beta};
  for (auto v : sc)
    if (!view_ok(*v, es)) return ZB_ERR_LAYOUT;
  if (!a->status) return ZB_ERR_LAYOUT;
  const bool state_only = (a->flags & ZB_FLAG_STATE_ONLY) != 0;
  if (!backward) {
    if (!state_only && !view_ok(a->y, e)) return ZB_ERR_LAYOUT;
  } else {
    if (!a->states && !state_only) return ZB_ERR_WORKSPACE;
    if (!view_ok(a->dy, e)) return ZB_ERR_LAYOUT;
    if (!state_only) {
      const zb_view* gv[] = {&a->dx, &a->dq, &a->dk, &a->dkp, &a->dxp};
      for (auto v : gv)
        if (!view_ok(*v, e)) return ZB_ERR_LAYOUT;
      const zb_view* gs[] = {&a->dadt, &a->dgamma, &a->dbeta};
      for (auto v : gs)
        if (!view_ok(*v, es)) return ZB_ERR_LAYOUT;
    }
  }
  return ZB_OK;
}

// Kernel family for these arguments.  The tensor-core family is used for everything it has
// both directions for (tc_has_backward); until then only for forwards that save no states,
// so the saved-state layout a backward reads always matches the forward that wrote it.
int make_plan(const zb_ssd_args* a, Plan* pl, bool stateless_forward) {
  const int64_t BH = a->B * a->H;
  if (tc_supported(a) && (tc_has_backward(a) || stateless_forward)) {
    pl->kind = kTc;
    pl->L = tc_chunk();
    pl->nc = (int)((a->T + pl->L - 1) / pl->L);
    pl->acc = 4;
    pl->states_bytes = tc_states_bytes(a);
    pl->sync_bytes = chain_sync_bytes(BH * (pl->nc + 1));
    pl->gchain_bytes = 0;
    pl->grp_bytes = 0;
    pl->tc_fwd_ws = tc_workspace_bytes(a, false);
    pl->tc_bwd_ws = tc_workspace_bytes(a, true);
    return ZB_OK;
  }
  const bool f64 = a->dtype == ZB_F64;
  const int L = simt_pick_chunk((int)a->P, (int)a->N, f64);
  if (L == 0) return ZB_ERR_UNSUPPORTED;
  pl->kind = kSimt;
  pl->L = L;
  pl->nc = (int)((a->T + L - 1) / L);
  pl->acc = f64 ? 8 : 4;
  const size_t slots = (size_t)BH * (pl->nc + 1) * (size_t)a->P * (size_t)a->N;
  pl->states_bytes = align_up(slots * pl->acc, 256);
  pl->sync_bytes = chain_sync_bytes(BH * (pl->nc + 1));
  pl->gchain_bytes = pl->states_bytes;
  pl->grp_bytes = (a->G != a->H) ? align_up((size_t)a->B * a->T * a->H * 3 * a->N * pl->acc, 256) : 0;
  pl->tc_fwd_ws = pl->tc_bwd_ws = 0;
  return ZB_OK;
}

View to_view(const zb_view& v) { return View{v.ptr, v.sb, v.st, v.sh}; }

// ZB_FLAG_SHIFTED: xp / kp are read from x / k one token earlier; give them x's and k's views
const zb_ssd_args* unshift(const zb_ssd_args* a, zb_ssd_args* tmp) {
  if (!a || !(a->flags & ZB_FLAG_SHIFTED)) return a;
  *tmp = *a;
  tmp->kp = tmp->k;
  tmp->xp = tmp->x;
  return tmp;
}

SimtParams simt_params(const zb_ssd_args* a, const Plan& pl) {
  SimtParams p;
  memset(&p, 0, sizeof(p));
  p.B = a->B; p.T = a->T; p.H = a->H; p.G = a->G; p.P = a->P; p.N = a->N;
  p.L = pl.L; p.nc = pl.nc; p.flags = a->flags;
  p.x = to_view(a->x); p.q = to_view(a->q); p.k = to_view(a->k); p.kp = to_view(a->kp); p.xp = to_view(a->xp);
  p.adt = to_view(a->adt); p.gamma = to_view(a->gamma); p.beta = to_view(a->beta);
  p.y = to_view(a->y);
  p.init = a->initial_state; p.fin = a->final_state;
  p.status = a->status;
  p.dy = to_view(a->dy); p.dfin = a->dfinal_state;
  p.dx = to_view(a->dx); p.dq = to_view(a->dq); p.dk = to_view(a->dk); p.dkp = to_view(a->dkp); p.dxp = to_view(a->dxp);
  p.dadt = to_view(a->dadt); p.dgamma = to_view(a->dgamma); p.dbeta = to_view(a->dbeta);
  p.dinit = a->dinitial_state;
  return p;
}

__global__ void state_combine_kernel(const float* s_prev, const float* decay, const float* f_prev, float* s_next,
                                     int64_t BH, int64_t PN) {
  const int64_t total = BH * PN;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    s_next[i] = decay[i / PN] * s_prev[i] + f_prev[i];
}

template <typename TS>
__global__ void total_decay_kernel(View adt, int64_t T, int64_t H, float* out) {
  const int64_t bh = blockIdx.x, b = bh / H, h = bh % H;
  double acc = 0.0;
  for (int64_t t = threadIdx.x; t < T; t += blockDim.x) acc += (double)ldv<float>(adt.row<TS>(b, t, h));
  __shared__ double red[32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    out[bh] = (float)exp(s);
  }
}

}  // namespace

extern "C" {

int zb_version(void) { return 100; }

const char* zb_strerror(int s) {
  switch (s) {
    case ZB_OK: return "ok";
    case ZB_ERR_SHAPE: return "bad shape (sequence length must be a multiple of chunk_size; H % G == 0; sizes > 0)";
    case ZB_ERR_DTYPE: return "unsupported dtype combination";
    case ZB_ERR_LAYOUT: return "bad layout (NULL or misaligned pointer)";
    case ZB_ERR_CUDA: return "CUDA error";
    case ZB_ERR_TIMEOUT: return "timed out waiting for the preceding chunk's state";
    case ZB_ERR_WORKSPACE: return "workspace or saved-states buffer missing, too small or misaligned";
    case ZB_ERR_UNSUPPORTED: return "sizes not supported by the kernels";
    case ZB_ERR_SCRATCH_LIMIT: return "call needs more scratch than the fixed no-alloc array (ZB_NOALLOC_SCRATCH_BYTES)";
    case ZB_ERR_INDEX: return "label outside [0, vocabulary size)";
    default: return "unknown status";
  }
}

const char* zb_last_cuda_error(void) { return g_cuda_err; }

size_t zb_ssd_states_bytes(const zb_ssd_args* a_) {
  zb_ssd_args tmp_;
  const zb_ssd_args* a = unshift(a_, &tmp_);
  if (validate(a, false) != ZB_OK && validate(a, true) != ZB_OK) {
    // shape/dtype check only: pointers may be unset when sizing
    if (!a || a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0) return 0;
    if (a->chunk_size <= 0 || a->T % a->chunk_size || a->H % a->G) return 0;
    if (!dtype_size(a->dtype) || !dtype_size(a->scalar_dtype)) return 0;
  }
  Plan pl;
  if (make_plan(a, &pl, false) != ZB_OK) return 0;
  return pl.states_bytes;
}

namespace {
// scratch a plan needs: [sync | TC ring] or [sync | SIMT chain (fwd) / gradient chain + groups (bwd)]
size_t plan_workspace(const Plan& pl, bool backward) {
  if (pl.kind == kTc) return pl.sync_bytes + (backward ? pl.tc_bwd_ws : pl.tc_fwd_ws);
  if (!backward) return pl.sync_bytes + pl.states_bytes;  // the chain lives here when no states buffer is given
  return pl.sync_bytes + pl.gchain_bytes + pl.grp_bytes;
}

// ---------------------------------------------------------------------------------------------
// Segmented long sequences.  With fewer (batch, head) chains than SMs, a long sequence would be
// handed chunk to chunk through one long chain per (batch, head).  Instead each sequence is viewed
// as M consecutive segments (M sequences of T/M tokens: a pure stride change when the batch
// dimension is contiguous), and the same linear algebra as context parallelism joins them:
//   forward : F_m, D_m = final state from zero and exp(sum adt) of segment m (state-only pass);
//             S_m = D_{m-1} S_{m-1} + F_{m-1} (combine kernel); full pass with initial states S_m.
//   backward: G_m = d(initial state of m) from segment m's own dy (state-only pass);
//             E_{m-1} = D_m E_m + G_m (combine kernel); full pass with final-state gradients E_m.
// The decision depends only on sizes and the input views, so forward and backward agree.
// When to segment: a chain hands its state on once per 64-token chunk, about 3 us per hand-off in
// each direction, so T / 64 hand-offs bound a call from below; the chunks' own work spreads over
// the SMs.  Measured on the layer shape (B x 24 heads x T 2048, one B200, fwd + bwd): unsegmented
// 197 / 220 / 341 us at B = 1 / 2 / 4, segmented into 8 / 4 / 4 segments 175 / 271 / 495 us.  The
// extra state-only pass and combine step pay only when there are fewer chains than about a
// quarter of the SMs.  How many segments: one chain per SM is enough; more only add segment
// boundaries (B1 x 24 heads x T 131072, chunk 128, fwd + bwd: 4 / 8 / 16 / 32 segments per
// sequence 7.61 / 5.88 / 6.14 / 6.62 ms).
constexpr int kSegChainsPerSm = 4;       // segment only while chains * 4 < SMs
constexpr int kSegMinChunks = 4;         // and keep at least four chunks per chain

bool batch_contiguous(const zb_view& v, int64_t T) { return v.sb == T * v.st; }

// streaming multiprocessors of the current device (cached per device)
int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int segments_for(const zb_ssd_args* a, const Plan& pl) {
  if (pl.kind != kTc || (a->flags & ZB_FLAG_SHIFTED)) return 1;  // a segment's row -1 is not zero
  const int64_t chains = a->B * a->H;
  if (chains * kSegChainsPerSm >= device_sms()) return 1;
  const zb_view* v[] = {&a->x, &a->q, &a->k, &a->kp, &a->xp, &a->adt, &a->gamma, &a->beta};
  for (auto x : v)
    if (!batch_contiguous(*x, a->T)) return 1;
  int M = 1;
  const int64_t sms = device_sms();
  while (chains * M < sms && pl.nc % (2 * M) == 0 && pl.nc / (2 * M) >= kSegMinChunks) M *= 2;
  return M;
}

zb_view seg_view(const zb_view& v, int64_t T, int M) {
  zb_view o = v;
  o.sb = (T / M) * v.st;
  return o;
}

// the arguments seen as B*M sequences of T/M tokens (views must be batch-contiguous)
bool seg_args(const zb_ssd_args* a, int M, bool backward, zb_ssd_args* s) {
  *s = *a;
  s->B = a->B * M;
  s->T = a->T / M;
  s->chunk_size = tc_chunk();
  zb_view* v[] = {&s->x, &s->q, &s->k, &s->kp, &s->xp, &s->adt, &s->gamma, &s->beta};
  for (auto x : v) *x = seg_view(*x, a->T, M);
  const bool state_only = (a->flags & ZB_FLAG_STATE_ONLY) != 0;
  if (!backward) {
    if (state_only) return true;
    if (!batch_contiguous(a->y, a->T)) return false;
    s->y = seg_view(a->y, a->T, M);
  } else {
    const zb_view* src[] = {&a->dy, &a->dx, &a->dq, &a->dk, &a->dkp, &a->dxp, &a->dadt, &a->dgamma, &a->dbeta};
    zb_view* dst[] = {&s->dy, &s->dx, &s->dq, &s->dk, &s->dkp, &s->dxp, &s->dadt, &s->dgamma, &s->dbeta};
    for (int i = 0; i < 9; ++i) {
      if (!batch_contiguous(*src[i], a->T)) return false;
      *dst[i] = seg_view(*src[i], a->T, M);
    }
  }
  return true;
}

struct SegLayout {
  size_t sync, ring, fg, d, se, total;  // byte offsets of each part, and the total
};

SegLayout seg_layout(const zb_ssd_args* a, int M) {
  const int64_t BHs = a->B * M * a->H, nc = a->T / M / tc_chunk();
  const size_t pn = (size_t)a->P * a->N * sizeof(float);
  SegLayout L;
  L.sync = 0;
  L.ring = chain_sync_bytes(BHs * (nc + 1));
  L.fg = L.ring + align_up((size_t)BHs * 2 * pn, 256);
  L.d = L.fg + align_up((size_t)BHs * pn, 256);
  L.se = L.d + align_up((size_t)BHs * sizeof(float), 256);
  L.total = L.se + align_up((size_t)BHs * pn, 256);
  return L;
}

// Combine kernels: one CTA row per (batch, head) and one thread per state element e.  The chain over
// the M segments is serial in its arithmetic only: each batch of kCombineBatch segments' F / G and D
// is loaded before any of them is used (the pointers are restrict-qualified), so a thread waits for
// one round of loads per batch instead of one per segment.
constexpr int kCombineBatch = 8;

// forward: segment initial states from `init` (or zero), F and D; writes the final state
__global__ void seg_combine_fwd_kernel(const float* __restrict__ init, const float* __restrict__ F,
                                       const float* __restrict__ D, float* __restrict__ S, float* __restrict__ fin,
                                       int H, int M, int64_t PN) {
  const int64_t e = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= PN) return;
  const int bh = blockIdx.x, b = bh / H, h = bh - b * H;
  float s = init ? init[(int64_t)bh * PN + e] : 0.f;
  for (int m0 = 0; m0 < M; m0 += kCombineBatch) {
    float f[kCombineBatch], d[kCombineBatch];
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      const int64_t idx = ((int64_t)b * M + m0 + u) * H + h;
      f[u] = (m0 + u < M) ? F[idx * PN + e] : 0.f;
      d[u] = (m0 + u < M) ? D[idx] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      if (m0 + u >= M) break;
      const int64_t idx = ((int64_t)b * M + m0 + u) * H + h;
      S[idx * PN + e] = s;
      s = d[u] * s + f[u];
    }
  }
  if (fin) fin[(int64_t)bh * PN + e] = s;
}

// backward: gradient w.r.t. each segment's final state, from `dfinal` (or zero), the segments' own
// initial-state gradients G and D; writes the gradient w.r.t. the initial state
__global__ void seg_combine_bwd_kernel(const float* __restrict__ dfinal, const float* __restrict__ G,
                                       const float* __restrict__ D, float* __restrict__ E, float* __restrict__ dinit,
                                       int H, int M, int64_t PN) {
  const int64_t e = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= PN) return;
  const int bh = blockIdx.x, b = bh / H, h = bh - b * H;
  float g = dfinal ? dfinal[(int64_t)bh * PN + e] : 0.f;
  for (int m1 = M; m1 > 0; m1 -= kCombineBatch) {  // segments m1-1 down to m1-kCombineBatch
    float gg[kCombineBatch], d[kCombineBatch];
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      const int m = m1 - 1 - u;
      const int64_t idx = ((int64_t)b * M + m) * H + h;
      gg[u] = (m >= 0) ? G[idx * PN + e] : 0.f;
      d[u] = (m >= 0) ? D[idx] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      const int m = m1 - 1 - u;
      if (m < 0) break;
      const int64_t idx = ((int64_t)b * M + m) * H + h;
      E[idx * PN + e] = g;
      g = d[u] * g + gg[u];
    }
  }
  if (dinit) dinit[(int64_t)bh * PN + e] = g;
}

int launch_total_decay(const zb_ssd_args* a, float* out, cudaStream_t s);

// segmented forward / backward (see above); `ws` holds SegLayout
int seg_fwd(const zb_ssd_args* a, int M, char* ws, cudaStream_t stream) {
  const SegLayout L = seg_layout(a, M);
  zb_ssd_args sa;
  if (!seg_args(a, M, false, &sa)) return ZB_ERR_LAYOUT;
  const int64_t BHs = sa.B * sa.H;
  const size_t sync_bytes = chain_sync_bytes(BHs * (sa.T / tc_chunk() + 1));
  float* F = reinterpret_cast<float*>(ws + L.fg);
  float* D = reinterpret_cast<float*>(ws + L.d);
  float* Sg = reinterpret_cast<float*>(ws + L.se);
  ChainSync sync{reinterpret_cast<unsigned int*>(ws), reinterpret_cast<int*>(ws + 256)};
  cudaError_t e = cudaMemsetAsync(ws, 0, sync_bytes, stream);
  if (e != cudaSuccess) return ZB_ERR_CUDA;
  zb_ssd_args st = sa;
  st.flags |= ZB_FLAG_STATE_ONLY;
  st.initial_state = nullptr;
  st.final_state = F;
  st.states = nullptr;
  int rc = tc_fwd(&st, sync, nullptr, ws + L.ring, stream);
  if (rc) return rc;
  if ((rc = launch_total_decay(&sa, D, stream))) return rc;
  const int64_t PN = a->P * a->N;
  const dim3 cgrid((unsigned)(a->B * a->H), (unsigned)((PN + 255) / 256));
  seg_combine_fwd_kernel<<<cgrid, 256, 0, stream>>>(static_cast<const float*>(a->initial_state), F, D, Sg,
                                                    static_cast<float*>(a->final_state), (int)a->H, M, PN);
  note_launches(1);
  if (a->flags & ZB_FLAG_STATE_ONLY) return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
  if ((e = cudaMemsetAsync(ws, 0, sync_bytes, stream)) != cudaSuccess) return ZB_ERR_CUDA;
  zb_ssd_args full = sa;
  full.initial_state = Sg;
  full.final_state = nullptr;
  return tc_fwd(&full, sync, a->states, ws + L.ring, stream);
}

int seg_bwd(const zb_ssd_args* a, int M, char* ws, cudaStream_t stream) {
  const SegLayout L = seg_layout(a, M);
  zb_ssd_args sa;
  if (!seg_args(a, M, true, &sa)) return ZB_ERR_LAYOUT;
  const int64_t BHs = sa.B * sa.H;
  const size_t sync_bytes = chain_sync_bytes(BHs * (sa.T / tc_chunk() + 1));
  float* G = reinterpret_cast<float*>(ws + L.fg);
  float* D = reinterpret_cast<float*>(ws + L.d);
  float* E = reinterpret_cast<float*>(ws + L.se);
  ChainSync sync{reinterpret_cast<unsigned int*>(ws), reinterpret_cast<int*>(ws + 256)};
  cudaError_t e = cudaMemsetAsync(ws, 0, sync_bytes, stream);
  if (e != cudaSuccess) return ZB_ERR_CUDA;
  zb_ssd_args st = sa;
  st.flags |= ZB_FLAG_STATE_ONLY;
  st.dfinal_state = nullptr;
  st.dinitial_state = G;
  int rc = tc_bwd(&st, sync, ws + L.ring, stream);
  if (rc) return rc;
  if ((rc = launch_total_decay(&sa, D, stream))) return rc;
  const int64_t PN = a->P * a->N;
  const dim3 cgrid((unsigned)(a->B * a->H), (unsigned)((PN + 255) / 256));
  seg_combine_bwd_kernel<<<cgrid, 256, 0, stream>>>(static_cast<const float*>(a->dfinal_state), G, D, E,
                                                    static_cast<float*>(a->dinitial_state), (int)a->H, M, PN);
  note_launches(1);
  if (a->flags & ZB_FLAG_STATE_ONLY) return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
  if ((e = cudaMemsetAsync(ws, 0, sync_bytes, stream)) != cudaSuccess) return ZB_ERR_CUDA;
  zb_ssd_args full = sa;
  full.dfinal_state = E;
  full.dinitial_state = nullptr;
  return tc_bwd(&full, sync, ws + L.ring, stream);
}
}  // namespace

namespace {
int launch_total_decay(const zb_ssd_args* a, float* out, cudaStream_t s) {
  const unsigned nb = (unsigned)(a->B * a->H);
  const View v = to_view(a->adt);
  switch (a->scalar_dtype) {
    case ZB_F32: total_decay_kernel<float><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_BF16: total_decay_kernel<__nv_bfloat16><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_F16: total_decay_kernel<__half><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_F64: total_decay_kernel<double><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    default: return ZB_ERR_DTYPE;
  }
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}
}  // namespace

size_t zb_ssd_workspace_bytes(const zb_ssd_args* a_, int backward) {
  zb_ssd_args tmp_;
  const zb_ssd_args* a = unshift(a_, &tmp_);
  if (!a || a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0) return 0;
  if (a->chunk_size <= 0 || a->T % a->chunk_size || a->H % a->G) return 0;
  if (!dtype_size(a->dtype) || !dtype_size(a->scalar_dtype)) return 0;
  Plan pl;
  if (make_plan(a, &pl, false) != ZB_OK) return 0;
  size_t need = plan_workspace(pl, backward != 0);
  int M = segments_for(a, pl);
  if (!backward) {  // a forward may run with or without a states buffer: cover both plans
    Plan p2;
    if (make_plan(a, &p2, true) == ZB_OK) {
      need = std::max(need, plan_workspace(p2, false));
      M = std::max(M, segments_for(a, p2));
    }
  }
  if (M > 1) need = std::max(need, seg_layout(a, M).total);
  return need;
}

int zb_ssd_fwd(const zb_ssd_args* a_, void* stream_) {
  zb_ssd_args tmp_;
  const zb_ssd_args* a = unshift(a_, &tmp_);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int rc = validate(a, false);
  if (rc) return rc;
  Plan pl;
  if ((rc = make_plan(a, &pl, a->states == nullptr))) return rc;
  const int M = segments_for(a, pl);
  const size_t need = M > 1 ? seg_layout(a, M).total : plan_workspace(pl, false);
  if (!a->workspace || a->workspace_bytes < need || reinterpret_cast<uintptr_t>(a->workspace) % 256) return ZB_ERR_WORKSPACE;
  if (a->states && reinterpret_cast<uintptr_t>(a->states) % 256) return ZB_ERR_WORKSPACE;
  char* ws = static_cast<char*>(a->workspace);
  if (M > 1) {
    rc = seg_fwd(a, M, ws, stream);
    if (rc == ZB_ERR_CUDA) return cuda_fail(cudaGetLastError());
    return rc;
  }
  cudaError_t e = cudaMemsetAsync(ws, 0, pl.sync_bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e);
  ChainSync sync{reinterpret_cast<unsigned int*>(ws), reinterpret_cast<int*>(ws + 256)};
  void* chain = a->states ? a->states : static_cast<void*>(ws + pl.sync_bytes);
  if (pl.kind == kTc) {
    rc = tc_fwd(a, sync, a->states, ws + pl.sync_bytes, stream);
  } else {
    SimtParams p = simt_params(a, pl);
    p.sync = sync;
    p.chain = chain;
    rc = simt_launch(p, a->dtype, a->scalar_dtype, false, stream);
  }
  if (rc == ZB_ERR_CUDA) return cuda_fail(cudaGetLastError());
  return rc;
}

int zb_ssd_bwd(const zb_ssd_args* a_, void* stream_) {
  zb_ssd_args tmp_;
  const zb_ssd_args* a = unshift(a_, &tmp_);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int rc = validate(a, true);
  if (rc) return rc;
  Plan pl;
  if ((rc = make_plan(a, &pl, false))) return rc;
  const int M = segments_for(a, pl);
  const size_t need = M > 1 ? seg_layout(a, M).total : plan_workspace(pl, true);
  if (!a->workspace || a->workspace_bytes < need || reinterpret_cast<uintptr_t>(a->workspace) % 256) return ZB_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(a->states) % 256) return ZB_ERR_WORKSPACE;
  char* ws = static_cast<char*>(a->workspace);
  if (M > 1) {
    rc = seg_bwd(a, M, ws, stream);
    if (rc == ZB_ERR_CUDA) return cuda_fail(cudaGetLastError());
    return rc;
  }
  cudaError_t e = cudaMemsetAsync(ws, 0, pl.sync_bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e);
  ChainSync sync{reinterpret_cast<unsigned int*>(ws), reinterpret_cast<int*>(ws + 256)};
  if (pl.kind == kTc) {
    rc = tc_bwd(a, sync, ws + pl.sync_bytes, stream);
  } else {
    SimtParams p = simt_params(a, pl);
    p.sync = sync;
    p.chain = a->states;
    p.gchain = ws + pl.sync_bytes;
    p.grp = pl.grp_bytes ? static_cast<void*>(ws + pl.sync_bytes + pl.gchain_bytes) : nullptr;
    rc = simt_launch(p, a->dtype, a->scalar_dtype, true, stream);
  }
  if (rc == ZB_ERR_CUDA) return cuda_fail(cudaGetLastError());
  return rc;
}

int zb_ssd_state_combine(const float* s_prev, const float* decay_prev, const float* f_prev, float* s_next, int64_t BH,
                         int64_t PN, void* stream) {
  if (!s_prev || !decay_prev || !f_prev || !s_next || BH <= 0 || PN <= 0) return ZB_ERR_LAYOUT;
  const int64_t total = BH * PN;
  const unsigned nb = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 8);
  state_combine_kernel<<<nb, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(s_prev, decay_prev, f_prev, s_next, BH, PN);
  note_launches(1);
  cudaError_t e = cudaPeekAtLastError();
  return e == cudaSuccess ? ZB_OK : cuda_fail(e);
}

int zb_ssd_total_decay(const zb_ssd_args* a, float* out, void* stream) {
  if (!a || !out || !a->adt.ptr || a->B <= 0 || a->T <= 0 || a->H <= 0) return ZB_ERR_LAYOUT;
  const unsigned nb = (unsigned)(a->B * a->H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const View v = to_view(a->adt);
  switch (a->scalar_dtype) {
    case ZB_F32: total_decay_kernel<float><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_BF16: total_decay_kernel<__nv_bfloat16><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_F16: total_decay_kernel<__half><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    case ZB_F64: total_decay_kernel<double><<<nb, 256, 0, s>>>(v, a->T, a->H, out); break;
    default: return ZB_ERR_DTYPE;
  }
  note_launches(1);
  cudaError_t e = cudaPeekAtLastError();
  return e == cudaSuccess ? ZB_OK : cuda_fail(e);
}

int zb_ssd_check_status(const int32_t* status, void* stream) {
  if (!status) return ZB_ERR_LAYOUT;
  int32_t h = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&h, status, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e);
  return h;
}

uint64_t zb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int zb_ssd_kernel_family(const zb_ssd_args* a_, int states_saved) {
  zb_ssd_args tmp_;
  const zb_ssd_args* a = unshift(a_, &tmp_);
  if (!a || a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0) return -1;
  if (a->chunk_size <= 0 || a->T % a->chunk_size || a->H % a->G) return -1;
  if (!dtype_size(a->dtype) || !dtype_size(a->scalar_dtype)) return -1;
  Plan pl;
  if (make_plan(a, &pl, states_saved == 0) != ZB_OK) return -1;
  return pl.kind == kTc ? 1 : 0;
}

}  // extern "C"
