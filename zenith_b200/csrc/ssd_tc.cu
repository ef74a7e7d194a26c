// Tensor-core path of the SSD chunked scan for bf16 vectors (P = 64, N = 64 or 128, fp32
// per-token scalars): tcgen05 MMAs with fp32 accumulators in TMEM, operands staged in shared
// memory by TMA (128-byte swizzle, no multicast).
//
// Forward, persistent, 128 TMEM columns and 68 KB (N = 128: 256 threads, 3 CTAs per SM) or 52 KB
// (N = 64: 128 threads, 4 CTAs per SM) of shared memory, so that several CTAs share an SM and run
// each other's dependent phases in between.  Per (batch, head, 64-token chunk):
//   MMA1  S    = Q [K;Kp]^T                M=64 (t)  N=128 (s|s')  K=N    lanes 0-15,  cols 0-127
//   K, Kp rows scaled in place by w g, w b (MMA1 is done with them)
//   MMA3  Sl_h = [wgK;wbKp]_h^T [X;Xp]     M=64 (n of half h) N=64 (p) K=128  lanes 16-31, cols 64h..
//   epilogue: Ps = (S * [g|b]_s * exp(c_t - c_s) masked to s <= t) -> registers -> bf16 over K|Kp
//   MMA2  Yi   = Ps [X;Xp]                 M=64 (t)  N=64 (p)  K=128    lanes 0-15, cols 0-63 (S consumed)
//   chain: wait for S_in[j]; S_in[j+1] = e^{c_L} S_in[j] + Sl -> ring slot; publish; S_in[j] bf16 -> smem
//   MMA4  Ye   = Q S_in[j]^T               M=64 (t)  N=64 (p)  K=N      lanes 0-15, cols 64-127
//   epilogue: y = Yi + e^{c_t} Ye -> bf16 -> TMA store
// The fp32 state hand-off lives in a two-slot ring per (batch, head) that stays in L2; the
// states the backward needs are saved in bf16 [B*H][nc][N][P].
#include <cuda.h>

#include <atomic>
#include <mutex>

#include "ssd_tc.h"
#include "ssd_kernels.h"
#include "umma.cuh"

namespace zb {

namespace {

constexpr int kL = 64;  // internal chunk length
constexpr int kP = 64;

// Per-chunk scalar block in shared memory (floats): [c | ec | w | wg | wb | g | b | es] (64 each),
// then at kScalFast a flag: 1 when every adt of the chunk lies in [-8, 0].  es_s = e^{c_r - c_s}
// with r the first token of s's 8-token block, so that the decay e^{c_t - c_s} = e^{c_t - c_r} es_s
// (t >= s) costs one exponential per (row, block) instead of one per element.  Under the flag c
// does not increase, so e^{c_t - c_r} <= 1 and 1 <= es_s <= e^{56}; where e^{c_t - c_r} underflows
// (below 1e-38) the true decay is below 1e-38 e^{56} ~ 2e-14, negligible beside the O(1) entries.
// Other chunks use the per-element exponential.
constexpr int kScal = 576;
constexpr int kScalEs = 448;
constexpr int kScalFast = 514;

// Shared memory of the forward.  After MMA3 the K|Kp block 0 holds the scores Ps [2][64 t][64 s]
// and (N = 128) block 1 the S_in image; after MMA4 the X tile holds the y tile.
template <int NS>
struct FwdSmem {
  static constexpr int QB = NS / 64;                      // 64-wide blocks along n
  static constexpr uint32_t Q = 0;                        // [QB][64 t][64 n]
  static constexpr uint32_t KK = Q + QB * 8192;           // [QB][K | Kp][64 s][64 n]
  static constexpr uint32_t XX = KK + QB * 16384;         // [X | Xp] [64 s][64 p]
  static constexpr uint32_t SIN = NS == 128 ? KK + 16384 : XX + 16384;  // S_in image [NS n][64 p]
  static constexpr uint32_t SCAL = NS == 128 ? XX + 16384 : SIN + NS * 128;
  // per chunk parity [c | ec | w | wg | wb | g | b] (64 floats each), then the next chunk's staged
  // adt, gamma, beta
  static constexpr uint32_t BAR = SCAL + (2 * kScal + 192) * 4;  // mbarriers: loads, MMA1, MMA3, MMA2 + MMA4
  static constexpr uint32_t MISC = BAR + 4 * 8;           // tmem base, first ticket, chain result, next ticket
  static constexpr uint32_t TOTAL = MISC + 16;
  static constexpr uint32_t ALLOC = TOTAL + 1024;         // slack to align the base to 1024
  static constexpr uint32_t LOAD_BYTES = QB * 8192 * 3 + 2 * 8192;
  static constexpr int CTAS_PER_SM = NS == 128 ? 3 : 4;   // shared memory: 70 KB / 54 KB per CTA
  static constexpr int THREADS = NS == 128 ? 256 : 128;   // registers: 80 / 128 per thread
  static constexpr int WPS = THREADS / 128;               // warps per TMEM sub-partition
};

struct TcFwdParams {
  CUtensorMap tq, tk, tkp, tx, txp;
  CUtensorMap ty;  // output, written by a TMA store from the staged tile
  int64_t B, T, H, G;
  int nc;
  const float* adt;
  const float* gamma;
  const float* beta;
  int64_t ssb, sst, ssh;  // strides of the three scalar views (all equal: checked on the host)
  int64_t asb, ast, ash, gsb, gst, gsh, bsb, bst, bsh;
  __nv_bfloat16* y;
  int64_t ysb, yst, ysh;
  const float* init;
  float* fin;
  __nv_bfloat16* states;  // [B*H][nc][N][P] or nullptr
  float* ring;            // [B*H][2][P][N]
  unsigned int* ticket;
  int* flags;             // [B*H][nc+1]
  int32_t* status;
  int shift;              // 1: tkp / txp map k / x, read one token earlier (row -1 is out of range: zeros)
  uint32_t band;          // chains per band of the ticket order (decode_ticket_banded)
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// 32 floats -> bf16 into chunks [c0, c0 + 4) of row r of a 128-byte-swizzled staging tile
__device__ __forceinline__ void stage_row32(unsigned char* tile, int r, int c0, const float* v) {
#pragma unroll
  for (int qd = 0; qd < 4; ++qd)
    *reinterpret_cast<uint4*>(tile + umma::sw128_offset(r, c0 + qd)) =
        make_uint4(pack_bf16(v[8 * qd], v[8 * qd + 1]), pack_bf16(v[8 * qd + 2], v[8 * qd + 3]),
                   pack_bf16(v[8 * qd + 4], v[8 * qd + 5]), pack_bf16(v[8 * qd + 6], v[8 * qd + 7]));
}

// 16 floats -> bf16 into chunks c0, c0 + 1 of row r of a 128-byte-swizzled staging tile
__device__ __forceinline__ void stage_row16(unsigned char* tile, int r, int c0, const float* v) {
#pragma unroll
  for (int qd = 0; qd < 2; ++qd)
    *reinterpret_cast<uint4*>(tile + umma::sw128_offset(r, c0 + qd)) =
        make_uint4(pack_bf16(v[8 * qd], v[8 * qd + 1]), pack_bf16(v[8 * qd + 2], v[8 * qd + 3]),
                   pack_bf16(v[8 * qd + 4], v[8 * qd + 5]), pack_bf16(v[8 * qd + 6], v[8 * qd + 7]));
}


// Two warps (token s = 0-63 per thread): the in-chunk cumulative sum c of adt and the per-token
// weights of one chunk, from its staged [adt | gamma | beta], into the scalar block sc
// (mamba3.py:40).  The two warps meet at named barrier 2.
__device__ __forceinline__ void chunk_scalars(float* sc, const float* nx, int s, int lane) {
  const float a = nx[s], gm = nx[64 + s], bt = nx[128 + s];
  float c = warp_incl_scan(a, lane);
  const bool pos = __any_sync(0xffffffffu, !(a <= 0.f && a >= -8.f));  // outside [-8, 0] (or NaN)
  if (s == 31) sc[31] = c;
  if (lane == 0) sc[512 + (s >> 5)] = pos ? 1.f : 0.f;
  asm volatile("bar.sync 2, 64;" ::: "memory");
  if (s >= 32) c += sc[31];
  if (s != 31) sc[s] = c;
  asm volatile("bar.sync 2, 64;" ::: "memory");
  const float w = expf(sc[63] - c);
  sc[64 + s] = expf(c);
  sc[128 + s] = w;
  sc[192 + s] = w * gm;
  sc[256 + s] = w * bt;
  sc[320 + s] = gm;
  sc[384 + s] = bt;
  sc[kScalEs + s] = expf(sc[s & ~7] - c);
  if (s == 0) sc[kScalFast] = (sc[512] + sc[513] > 0.f) ? 0.f : 1.f;
}

// Loads of one chunk's operands (Q, K | Kp, X | Xp), completing on one mbarrier.
// K | Kp block qb (n in [64 qb, 64 qb + 64))
__device__ __forceinline__ void fwd_load_kk_block(const TcFwdParams& p, unsigned char* sKK, uint64_t* bar, const UnitIdx& u,
                                                  int qb) {
  const int t0 = u.chunk * kL;
  umma::tma_load_4d(sKK + qb * 16384, &p.tk, bar, qb * 64, u.g, t0, u.b);
  umma::tma_load_4d(sKK + qb * 16384 + 8192, &p.tkp, bar, qb * 64, u.g, t0 - p.shift, u.b);
}
template <int NS>
__device__ __forceinline__ void fwd_load_kk(const TcFwdParams& p, unsigned char* sKK, uint64_t* bar, const UnitIdx& u) {
#pragma unroll
  for (int qb = 0; qb < NS / 64; ++qb) fwd_load_kk_block(p, sKK, bar, u, qb);
}
__device__ __forceinline__ void fwd_load_x(const TcFwdParams& p, unsigned char* sX, unsigned char* sXp, uint64_t* bar,
                                           const UnitIdx& u) {
  umma::tma_load_4d(sX, &p.tx, bar, 0, u.h, u.chunk * kL, u.b);
  umma::tma_load_4d(sXp, &p.txp, bar, 0, u.h, u.chunk * kL - p.shift, u.b);
}
template <int NS>
__device__ __forceinline__ void fwd_load_q(const TcFwdParams& p, unsigned char* sQ, uint64_t* bar, const UnitIdx& u) {
#pragma unroll
  for (int qb = 0; qb < NS / 64; ++qb) umma::tma_load_4d(sQ + qb * 8192, &p.tq, bar, qb * 64, u.g, u.chunk * kL, u.b);
}
// token s of a chunk: adt, gamma, beta -> dst[s], dst[64 + s], dst[128 + s] (asynchronous copies)
__device__ __forceinline__ void fwd_prefetch_scalars(const TcFwdParams& p, const UnitIdx& u, int s, float* dst) {
  const int t = u.chunk * kL + s;
  umma::cp_async4(dst + s, p.adt + (u.b * p.asb + t * p.ast + u.h * p.ash));
  umma::cp_async4(dst + 64 + s, p.gamma + (u.b * p.gsb + t * p.gst + u.h * p.gsh));
  umma::cp_async4(dst + 128 + s, p.beta + (u.b * p.bsb + t * p.bst + u.h * p.bsh));
  umma::cp_async_commit();
}

// Persistent: CTAS_PER_SM CTAs per SM walk the chunks in ticket order (chunk-major).  Each CTA
// takes its tickets in increasing order and a chunk only waits on a lower ticket, so the lowest
// unfinished ticket always belongs to a CTA that can run it.  The next chunk's operands load as
// the current chunk's tiles free (Q and K | Kp block 0 after MMA4, the rest once the y tile and
// the saved state have left shared memory), and warps 0-1 prepare the next chunk's scalars at the
// end of the current one.  Warp w reads TMEM sub-partition w % 4; with 8 warps (N = 128) the
// epilogues split their columns by w / 4.  Thread 0 issues the MMAs; the last warp's lane 0 issues
// the TMA and bulk copies.
template <int NS>
__global__ void __launch_bounds__(FwdSmem<NS>::THREADS, FwdSmem<NS>::CTAS_PER_SM)
    ssd_fwd_tc_kernel(const __grid_constant__ TcFwdParams p) {
  using S = FwdSmem<NS>;
  constexpr int QB = S::QB, WPS = S::WPS, ISS = S::THREADS - 32;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = sm + S::Q;
  unsigned char* sKK = sm + S::KK;
  unsigned char* sPs = sm + S::KK;   // scores, over K|Kp block 0 once MMA3 is done
  unsigned char* sX = sm + S::XX;
  unsigned char* sXp = sm + S::XX + 8192;
  unsigned char* sY = sm + S::XX;    // y tile, over X once MMA2 and MMA4 are done
  unsigned char* sSin = sm + S::SIN;
  float* s_scal = reinterpret_cast<float*>(sm + S::SCAL);  // [2 parity][c | ec | w | wg | wb | g | b]
  float* s_nx = s_scal + 2 * kScal;                            // next chunk's [adt | gamma | beta]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BAR);
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + S::MISC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, hw = warp >> 2;  // TMEM sub-partition, column share
  const bool hiL = lane >= 16;
  const int64_t total = p.B * p.H * p.nc;
  if (tid == 0) {
    misc[1] = atomicAdd(p.ticket, 1u);
    for (int i = 0; i < 4; ++i) umma::mbar_init(&bars[i], 1);
    umma::mbar_fence_init();
  }
  __syncwarp();  // lane 0 of warp 0 rejoins before the warp-collective allocation
  if (warp == 0) {
    umma::tmem_alloc(&misc[0], 128);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = misc[0];
  const uint32_t tlane = (uint32_t)(32 * sp) << 16;  // this warp's TMEM sub-partition
  uint32_t cur = misc[1];
  if (cur < total) {
    const UnitIdx u0 = decode_ticket_banded(cur, p.B, p.H, p.G, p.nc, p.band);
    if (tid == ISS) {
      umma::mbar_arrive_expect_tx(&bars[0], S::LOAD_BYTES);
      fwd_load_q<NS>(p, sQ, &bars[0], u0);
      fwd_load_kk<NS>(p, sKK, &bars[0], u0);
      fwd_load_x(p, sX, sXp, &bars[0], u0);
    }
    if (tid < 64) {
      fwd_prefetch_scalars(p, u0, tid, s_nx);
      umma::cp_async_wait_all();
      chunk_scalars(s_scal, s_nx, tid, lane);
    }
  }

  for (uint32_t it = 0; cur < total; ++it) {
    const uint32_t par = it & 1;  // parity of this chunk's barriers (each completes once per chunk)
    const UnitIdx u = decode_ticket_banded(cur, p.B, p.H, p.G, p.nc, p.band);
    const int j = u.chunk;
    const int64_t bh = u.bh;
    const int t0 = j * kL;
    int* flags = p.flags + bh * (p.nc + 1);
    uint32_t nx = 0, nxt = 0;
    if (tid == 0) nx = atomicAdd(p.ticket, 1u);  // the next ticket, published to the CTA at the chain
    // this chunk's scalars (mamba3.py:40) were prepared at the end of the previous one
    const float* s_c = s_scal + par * kScal;
    const float* s_ec = s_c + 64;
    const float* s_wg = s_c + 192;
    const float* s_wb = s_c + 256;
    const float* s_g = s_c + 320;
    const float* s_b = s_c + 384;
    const bool load_ok = umma::mbar_wait(&bars[0], par, p.status);
    bool ok = __syncthreads_and(load_ok);
    const float a_chunk = expf(s_c[63]);

    if (ok) {
      // MMA1: S = Q [K;Kp]^T
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t q0 = umma::smem_u32(sQ), kk0 = umma::smem_u32(sKK);
        constexpr uint32_t id1 = umma::idesc_bf16(64, 128, false, false);
#pragma unroll
        for (int ks = 0; ks < NS / 16; ++ks) {
          const uint32_t qb = ks >> 2, kin = ks & 3;
          umma::mma_bf16(tmem, umma::desc_sw128(q0 + qb * 8192 + kin * 32, 16, 1024),
                         umma::desc_sw128(kk0 + qb * 16384 + kin * 32, 16, 1024), id1, ks > 0);
        }
        umma::mma_commit(&bars[1]);
      }
      ok = __syncthreads_and(umma::mbar_wait(&bars[1], par, p.status));
    }
    constexpr int NPC = 8 / WPS;   // 16-column pieces of S per warp
    uint32_t pk[NPC / 2][8];       // this warp's Ps values (bf16 pairs) until K|Kp is free
    if (ok) {
      umma::fence_after_sync();
      // MMA1 is done with K|Kp: scale them in place, K rows s by w_s g_s and Kp rows by w_s b_s (for
      // MMA3).  A 16-byte chunk at byte offset o of a 64 x 64 tile lies in row (o mod 8192) / 128.
      for (uint32_t off = (uint32_t)tid * 16u; off < (uint32_t)QB * 16384u; off += S::THREADS * 16u) {
        const float f = ((off >> 13) & 1u) ? s_wb[(off & 8191u) >> 7] : s_wg[(off & 8191u) >> 7];
        const uint4 v = *reinterpret_cast<const uint4*>(sKK + off);
        uint4 o;
        float2 e;
        e = unpack_bf16(v.x); o.x = pack_bf16(e.x * f, e.y * f);
        e = unpack_bf16(v.y); o.y = pack_bf16(e.x * f, e.y * f);
        e = unpack_bf16(v.z); o.z = pack_bf16(e.x * f, e.y * f);
        e = unpack_bf16(v.w); o.w = pack_bf16(e.x * f, e.y * f);
        *reinterpret_cast<uint4*>(sKK + off) = o;
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      // MMA3: the chunk state, one M=64 product per 64-wide half of n, into lanes 16-31
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t kk0 = umma::smem_u32(sKK), x0 = umma::smem_u32(sX), xp0 = umma::smem_u32(sXp);
        constexpr uint32_t id3 = umma::idesc_bf16(64, 64, true, true);
#pragma unroll
        for (int hf = 0; hf < QB; ++hf) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t part = ks >> 2, kin = ks & 3;
            umma::mma_bf16(tmem + (16u << 16) + 64 * hf,
                           umma::desc_sw128(kk0 + hf * 16384 + part * 8192 + kin * 2048, 16384, 1024),
                           umma::desc_sw128((part ? xp0 : x0) + kin * 2048, 8192, 1024), id3, ks > 0);
          }
        }
        umma::mma_commit(&bars[2]);
      }
      // scores -> registers, 16 columns at a time while MMA3 runs.  TMEM gives lane l < 16 of the
      // warp the S row t = 16 sp + l; it keeps columns 0-7 of the piece and hands columns 8-15 to
      // lane l + 16 (one shuffle each).  Piece k (of 8): half k / 4 (0: K with gamma, 1: Kp with
      // beta), columns 16 (k % 4) of that half; warp w takes pieces [NPC (w / 4), NPC (w / 4 + 1)).
      {
        const int t = 16 * sp + (lane & 15);
        const float ct = s_c[t];
        const float* s_es = s_c + kScalEs;
        const bool fastm = s_c[kScalFast] != 0.f;
        // decay e^{c_t - c_s}: a lane's 8 columns of a piece are one 8-token block, factorised when
        // the chunk allows it (chunk_scalars)
        auto scores = [&](auto decay) {
#pragma unroll
          for (int pi = 0; pi < NPC; ++pi) {
            const int pc = hw * NPC + pi, half = pc >> 2;
            const float* coef = half ? s_b : s_g;
            const float et = fastm ? __expf(ct - s_c[16 * (pc & 3) + (hiL ? 8 : 0)]) : 0.f;
            float v[16];
            umma::tmem_ld16(tmem + tlane + pc * 16, v);
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              const float r0 = __shfl_xor_sync(0xffffffffu, v[8 + i], 16);
              const float r1 = __shfl_xor_sync(0xffffffffu, v[9 + i], 16);
              const int s0 = (pc & 3) * 16 + (hiL ? 8 : 0) + i;
              const float a0 = hiL ? r0 : v[i], a1 = hiL ? r1 : v[i + 1];
              const float v0 = (s0 <= t) ? a0 * coef[s0] * decay(et, s0) : 0.f;
              const float v1 = (s0 + 1 <= t) ? a1 * coef[s0 + 1] * decay(et, s0 + 1) : 0.f;
              pk[pi >> 1][(pi & 1) * 4 + (i >> 1)] = pack_bf16(v0, v1);
            }
          }
        };
        if (fastm)
          scores([&](float et, int s0) { return et * s_es[s0]; });
        else
          scores([&](float, int s0) { return __expf(ct - s_c[s0]); });
      }
      ok = __syncthreads_and(umma::mbar_wait(&bars[2], par, p.status));  // MMA3 done: K|Kp free
      if (ok) {
        // Ps (bf16, K-major [2][64 t][64 s]) over K|Kp block 0: piece k's 8 columns of this lane are
        // 16-byte chunk 2 (k % 4) + (lane >= 16) of row t in half k / 4
        const int t = 16 * sp + (lane & 15);
#pragma unroll
        for (int pi = 0; pi < NPC; ++pi) {
          const int pc = hw * NPC + pi;
          const uint32_t* w = &pk[pi >> 1][(pi & 1) * 4];
          *reinterpret_cast<uint4*>(sPs + (pc >> 2) * 8192 + umma::sw128_offset(t, 2 * (pc & 3) + (hiL ? 1 : 0))) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    if (ok) {
      umma::fence_after_sync();
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        umma::fence_after_sync();
        // MMA2: Yi = Ps [X;Xp] into lanes 0-15, cols 0-63 (the scores' TMEM has been read)
        const uint32_t ps0 = umma::smem_u32(sPs), x0 = umma::smem_u32(sX), xp0 = umma::smem_u32(sXp);
        constexpr uint32_t id2 = umma::idesc_bf16(64, 64, false, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t part = ks >> 2, kin = ks & 3;
          umma::mma_bf16(tmem, umma::desc_sw128(ps0 + part * 8192 + kin * 32, 16, 1024),
                         umma::desc_sw128((part ? xp0 : x0) + kin * 2048, 8192, 1024), id2, ks > 0);
        }
        misc[3] = nx;
      }
      // thread 32 waits for the preceding chunk's hand-off while thread 0 issues MMA2
      if (tid == 32) misc[2] = (j == 0) ? kFlagReady : wait_flag(&flags[j], p.status);
      __syncthreads();
      ok = misc[2] == kFlagReady;
      nxt = misc[3];
      if (!ok) {  // MMA2 must finish before TMEM is freed
        if (tid == 0) umma::mma_commit(&bars[3]);
        umma::mbar_wait(&bars[3], par, p.status);
      }
    }
    if (ok) {
      // state hand-off: S_in[j+1] = e^{c_L} S_in[j] + S_loc (mamba3.py:52).  Lanes 16-31 hold the
      // rows n = 64 h + 16 sp + lane - 16 of S_loc (half h); blocks of 16 columns p split over the
      // warps of a sub-partition, and within a block lane l < 16 takes columns 8-15 of lane l + 16's
      // row (one shuffle each).  A thread's ring loads of a batch of blocks are issued before any of
      // the batch's stores.
      // Ring slots are [p/4][n][4]; the caller's initial and final states are [p][n].  S_in[j] also
      // goes to shared memory in bf16 (the B operand of MMA4 and the saved state).
      const int64_t PN = (int64_t)kP * NS;
      const float4* ring_in = reinterpret_cast<const float4*>(p.ring + (bh * 2 + (j & 1)) * PN);
      float4* ring_out = reinterpret_cast<float4*>(p.ring + (bh * 2 + ((j + 1) & 1)) * PN);
      float* fin = (j == p.nc - 1 && p.fin) ? p.fin + bh * PN : nullptr;
      const float* init = p.init ? p.init + bh * PN : nullptr;
      constexpr int NP = 4 * QB / WPS;  // (half, 16-column block) pairs per warp
      constexpr int NBATCH = NP;  // every pair's ring loads in flight together (one L2 round trip)
      const int hs = hiL ? 0 : 1;       // which 8 columns of a block this lane takes
#pragma unroll
      for (int b0 = 0; b0 < NP; b0 += NBATCH) {
        float4 rin[NBATCH][2];
#pragma unroll
        for (int bi = 0; bi < NBATCH; ++bi) {
          const int pair = hw * NP + b0 + bi, hf = pair >> 2, pc = pair & 3;
          const int n = 64 * hf + 16 * sp + (lane & 15), p0 = 16 * pc + 8 * hs;
          if (j == 0) {
            float iv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) iv[i] = init ? __ldcg(init + (p0 + i) * NS + n) : 0.f;
            rin[bi][0] = make_float4(iv[0], iv[1], iv[2], iv[3]);
            rin[bi][1] = make_float4(iv[4], iv[5], iv[6], iv[7]);
          } else {
            rin[bi][0] = __ldcg(ring_in + (p0 / 4) * NS + n);
            rin[bi][1] = __ldcg(ring_in + (p0 / 4 + 1) * NS + n);
          }
        }
#pragma unroll
        for (int bi = 0; bi < NBATCH; ++bi) {
          const int pair = hw * NP + b0 + bi, hf = pair >> 2, pc = pair & 3;
          const int n = 64 * hf + 16 * sp + (lane & 15), p0 = 16 * pc + 8 * hs;
          float sl[16];
          umma::tmem_ld16(tmem + tlane + 64 * hf + 16 * pc, sl);
          float mine[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float r = __shfl_xor_sync(0xffffffffu, sl[8 + i], 16);
            mine[i] = hiL ? sl[i] : r;
          }
          const float sin[8] = {rin[bi][0].x, rin[bi][0].y, rin[bi][0].z, rin[bi][0].w,
                                rin[bi][1].x, rin[bi][1].y, rin[bi][1].z, rin[bi][1].w};
          float so[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) so[i] = a_chunk * sin[i] + mine[i];
          ring_out[(p0 / 4) * NS + n] = make_float4(so[0], so[1], so[2], so[3]);
          ring_out[(p0 / 4 + 1) * NS + n] = make_float4(so[4], so[5], so[6], so[7]);
          if (fin) {
#pragma unroll
            for (int i = 0; i < 8; ++i) fin[(p0 + i) * NS + n] = so[i];
          }
          *reinterpret_cast<uint4*>(sSin + umma::sw128_offset(n, p0 / 8)) =
              make_uint4(pack_bf16(sin[0], sin[1]), pack_bf16(sin[2], sin[3]), pack_bf16(sin[4], sin[5]),
                         pack_bf16(sin[6], sin[7]));
        }
      }
      // one barrier orders every thread's ring writes before thread 32's release (cumulative) and the
      // staged S_in before MMA4; the release, which waits for the ring writes to land, is kept off
      // the MMA issuer
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 32) st_release(&flags[j + 1], kFlagReady);
      if (tid == ISS && p.states) {
        // the saved state is the shared-memory image itself (bf16, 128-byte swizzle), so the
        // backward can bulk-copy it back into place
        umma::bulk_store(reinterpret_cast<unsigned char*>(p.states) + (bh * p.nc + j) * (int64_t)NS * 128, sSin,
                         NS * 128);
        umma::bulk_commit();
      }
      if (tid == 0) {
        umma::fence_after_sync();
        // MMA4: Ye = Q S_in^T into lanes 0-15, cols 64-127
        const uint32_t q0 = umma::smem_u32(sQ), sin0 = umma::smem_u32(sSin);
        constexpr uint32_t id4 = umma::idesc_bf16(64, 64, false, true);
#pragma unroll
        for (int ks = 0; ks < NS / 16; ++ks) {
          const uint32_t qb = ks >> 2, kin = ks & 3;
          umma::mma_bf16(tmem + 64, umma::desc_sw128(q0 + qb * 8192 + kin * 32, 16, 1024),
                         umma::desc_sw128(sin0 + ks * 2048, 8192, 1024), id4, ks > 0);
        }
        umma::mma_commit(&bars[3]);
      }
      if (tid < 64 && nxt < total) fwd_prefetch_scalars(p, decode_ticket_banded(nxt, p.B, p.H, p.G, p.nc, p.band), tid, s_nx);
      ok = __syncthreads_and(umma::mbar_wait(&bars[3], par, p.status));
    } else if (tid == 0) {
      st_release(&flags[j + 1], kFlagAbort);
    }
    if (ok) {
      umma::fence_after_sync();
      // MMA2 and MMA4 are done with Q and with Ps (K|Kp block 0): the next chunk's Q and first K|Kp
      // block start loading
      const UnitIdx nu = decode_ticket_banded(nxt < total ? nxt : 0, p.B, p.H, p.G, p.nc, p.band);
      if (tid == ISS && nxt < total) {
        umma::mbar_arrive_expect_tx(&bars[0], S::LOAD_BYTES);
        fwd_load_q<NS>(p, sQ, &bars[0], nu);
        fwd_load_kk_block(p, sKK, &bars[0], nu, 0);
      }
      // y = Yi + e^{c_t} Ye (mamba3.py:55): lanes 0-15 hold row t = 16 sp + lane; 16 columns at a
      // time, staged as a bf16 tile over X
      const int t = 16 * sp + (lane & 15);
      const float ect = s_ec[t];
#pragma unroll
      for (int qi = 0; qi < 4 / WPS; ++qi) {
        const int q = hw * (4 / WPS) + qi;
        float yi[16], ye[16];
        umma::tmem_ld16x2(tmem + tlane + 16 * q, tmem + tlane + 64 + 16 * q, yi, ye);
        if (!hiL) {
#pragma unroll
          for (int i = 0; i < 16; ++i) yi[i] += ect * ye[i];
          stage_row16(sY, t, 2 * q, yi);
        }
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == ISS) {
        umma::tma_store_4d(&p.ty, sY, 0, u.h, t0, u.b);
        umma::bulk_commit();
        // the y tile and the saved state leave shared memory, then the rest of the operands load
        umma::bulk_wait_read();
        if (nxt < total) {
#pragma unroll
          for (int qb = 1; qb < QB; ++qb) fwd_load_kk_block(p, sKK, &bars[0], nu, qb);
          fwd_load_x(p, sX, sXp, &bars[0], nu);
        }
      }
      if (tid < 64 && nxt < total) {  // the next chunk's scalars
        umma::cp_async_wait_all();
        chunk_scalars(s_scal + (par ^ 1) * kScal, s_nx, tid, lane);
      }
    }
    umma::fence_before_sync();
    __syncthreads();  // every read of this chunk's tiles, scalars and TMEM columns is done
    if (!ok) {
      // leave after an error: the ticket already taken is aborted (its loads were never issued)
      if (tid == 0 && nx < total) {
        const UnitIdx cn = decode_ticket_banded(nx, p.B, p.H, p.G, p.nc, p.band);
        st_release(&p.flags[cn.bh * (p.nc + 1) + cn.chunk + 1], kFlagAbort);
      }
      break;
    }
    umma::fence_after_sync();
    cur = nxt;
  }
  if (tid == ISS) umma::bulk_wait_all();  // staged tiles must be read out before exit
  if (tid < 64) umma::cp_async_wait_all();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------------------------------------
// backward
//
// Persistent CTAs (one per SM) take the (batch, head, chunk) units in reverse chunk order, 512
// threads, 512 TMEM columns.
//   MMA b  S      = Q [K;Kp]^T          M=64  N=128 K=N   -> R0 lanes +0
//   MMA a  dA     = dY [X;Xp]^T         M=64  N=128 K=64  -> R0 lanes +16
//   MMA g  dSl'   = Q^T dYe             M=N   N=64  K=64  -> R4     (dYe = e^{c_t} dY)
//   MMA h  Ye     = Q S_in^T            M=64  N=64  K=N   -> R1 lanes +16
//   MMA d  dQ     = dYe S_in            M=64  N=N   K=64  -> R1 lanes +0
//   side by side once those are done:
//     warps 0-7:  epilogue: A=S g M, Ap, E=dA M, Eg=E g, ... -> [A|Ap], [Eg|Epb] (bf16) and
//                 dc/dgamma/dbeta sums; then thread 0 issues
//       MMA c  dXc    = [A|Ap]^T dY         M=128 N=64  K=64  -> R2
//       MMA d  dQ    += [Eg|Epb] [K;Kp]     M=64  N=N   K=128 -> R1 lanes +0
//       MMA e  dK     = [Eg|Epb]^T Q        M=128 N=N   K=64  -> R0
//     warps 8-15: chain: wait for Gn = G[j+1]; G[j] = dSl'^T + e^{c_L} Gn -> ring; publish; Gn -> smem
//   MMA e  dK    += [wgX;wbXp] Gn       M=128 N=N   K=64  -> R0
//   MMA f  U      = [K;Kp] Gn^T         M=128 N=64  K=N   -> R3
//   epilogue: dx = dXc + w g U, dk, dq, per-token scalars, reverse cumsum -> dadt
// TMEM: R0 [0,128) R1 [128,256) R2 [256,320) R3 [320,384) R4 [384,448).

template <int NS>
struct BwdSmem {
  static constexpr int QB = NS / 64;
  // one input stage (two of them: the next chunk's operands land while this one is worked on)
  static constexpr uint32_t Q = 0;                  // [QB][64 t][64 n]; at the end the dq staging tile
  static constexpr uint32_t KK = Q + QB * 8192;     // [QB][K | Kp]; at the end the dk | dkp staging tiles
  static constexpr uint32_t XX = KK + QB * 16384;   // [X | Xp]  (128 rows); at the end dx | dxp
  static constexpr uint32_t DY = XX + 16384;
  static constexpr uint32_t SIN = DY + 8192;        // [NS n][64 p]
  static constexpr uint32_t STAGE = SIN + NS * 128;
  // shared work tiles, reused phase by phase
  static constexpr uint32_t W = 2 * STAGE;          // dYe -> [A | Ap] -> [wgX | wbXp]
  static constexpr uint32_t E = W + 16384;          // [Eg | Epb] -> Gn [NS n][64 p]
  // per-chunk scalars [c | ec | w | wg wb | g | b] (64 floats each), one block per chunk parity,
  // then the next chunk's staged [adt | gamma | beta]
  static constexpr uint32_t SCAL = E + 16384;
  static constexpr uint32_t RED = SCAL + (2 * kScal + 192) * 4;
  // RED: rowZ[4][64] | colZ[4][128] | colE[4][128] | xu[4][128] | dcint[2][64] | da[16] | tmp[8] | pre[3][64]
  static constexpr uint32_t RED_FLOATS = 256 + 512 + 512 + 512 + 128 + 16 + 8 + 192;
  static constexpr uint32_t BAR = RED + RED_FLOATS * 4;  // stage loads [2], MMA groups 1-3, hand-off and epilogue warps
  static constexpr uint32_t MISC = BAR + 7 * 8;          // tmem base, ticket, hand-off failures, next ticket
  static constexpr uint32_t TOTAL = MISC + 16;
  static constexpr uint32_t ALLOC = TOTAL + 1024;
  static_assert(STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
};

struct TcBwdParams {
  CUtensorMap tq, tk, tkp, tx, txp, tdy;
  CUtensorMap tdq, tdk, tdkp, tdx, tdxp;  // outputs, written by TMA stores from staged tiles
  int64_t B, T, H, G;
  int nc;
  const float* adt;
  const float* gamma;
  const float* beta;
  int64_t asb, ast, ash, gsb, gst, gsh, bsb, bst, bsh;
  const __nv_bfloat16* states;  // [B*H][nc] images of S_in (swizzled [N][P] bf16)
  const float* dfin;
  float* dinit;
  float* ring;                  // [B*H][2][P][N]
  __nv_bfloat16 *dx, *dxp, *dq, *dk, *dkp;
  int64_t dxsb, dxst, dxsh, dxpsb, dxpst, dxpsh, dqsb, dqst, dqsh, dksb, dkst, dksh, dkpsb, dkpst, dkpsh;
  float *dadt, *dgamma, *dbeta;
  int64_t dasb, dast, dash, dgsb, dgst, dgsh, dbsb, dbst, dbsh;
  unsigned int* ticket;
  int* flags;
  int32_t* status;
  int shift;  // as in TcFwdParams
};

constexpr int kBwdThreads = 512;

// scale each 128-byte row r of a bf16 tile by f[r] (rows = bytes / 128), src -> dst
__device__ __forceinline__ void scale_rows(const unsigned char* src, unsigned char* dst, uint32_t bytes, const float* f,
                                           int tid) {
  for (uint32_t off = (uint32_t)tid * 16u; off < bytes; off += kBwdThreads * 16u) {
    const float s = f[off >> 7];
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    uint4 o;
    float2 e;
    e = unpack_bf16(v.x); o.x = pack_bf16(e.x * s, e.y * s);
    e = unpack_bf16(v.y); o.y = pack_bf16(e.x * s, e.y * s);
    e = unpack_bf16(v.z); o.z = pack_bf16(e.x * s, e.y * s);
    e = unpack_bf16(v.w); o.w = pack_bf16(e.x * s, e.y * s);
    *reinterpret_cast<uint4*>(dst + off) = o;
  }
}

// v[i] (i < 16) is this lane's value in column i; the 16 lanes of each half-warp hold 16 rows.
// Returns the sum over those 16 rows of column (lane % 16) (reduce-scatter: 15 shuffles).
__device__ __forceinline__ float colsum16(float (&v)[16], int lane) {
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
    const bool hi = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = hi ? v[i] : v[i + w];
      const float keep = hi ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

// 8 consecutive bf16 of row r (16-byte chunk c) of a swizzled tile, as floats
__device__ __forceinline__ void load_chunk(const unsigned char* tile, int r, int c, float (&o)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(tile + umma::sw128_offset(r, c));
  float2 e;
  e = unpack_bf16(v.x); o[0] = e.x; o[1] = e.y;
  e = unpack_bf16(v.y); o[2] = e.x; o[3] = e.y;
  e = unpack_bf16(v.z); o[4] = e.x; o[5] = e.y;
  e = unpack_bf16(v.w); o[6] = e.x; o[7] = e.y;
}

// Persistent: one CTA per SM walks the chunks in ticket order (reverse chunk order), 512 threads.
// While a chunk is worked on, the next ticket's operands load into the other input stage.  Each
// CTA takes its tickets in increasing order and a chunk only waits on a lower ticket, so the
// lowest unfinished ticket always belongs to a CTA that can run it: no deadlock.
// The lane-parallel epilogues split four ways per TMEM sub-partition (warp w reads the lanes of
// sub-partition w % 4; w / 4 picks a column quarter).
struct BwdChunk {
  int j, b, h, g, t0;
  int64_t bh;
};

__device__ __forceinline__ BwdChunk bwd_chunk(const TcBwdParams& p, uint32_t tk) {
  const UnitIdx u = decode_ticket(tk, p.B, p.H, p.G);
  BwdChunk c;
  c.j = p.nc - 1 - u.chunk;
  c.bh = u.bh;
  c.b = u.b;
  c.h = u.h;
  c.g = u.g;
  c.t0 = c.j * kL;
  return c;
}

// one chunk's operands -> an input stage: Q, [K | Kp], [X | Xp], dY (TMA) and the saved S_in image
// (bulk copy), all completing on the stage's mbarrier
template <int NS>
__device__ __forceinline__ void bwd_issue_loads(const TcBwdParams& p, unsigned char* st, uint64_t* bar,
                                                const BwdChunk& c) {
  using S = BwdSmem<NS>;
  constexpr uint32_t kLoadBytes = S::QB * 8192 * 3 + 3 * 8192 + NS * 128;
  umma::mbar_arrive_expect_tx(bar, kLoadBytes);
#pragma unroll
  for (int qb = 0; qb < S::QB; ++qb) {
    umma::tma_load_4d(st + S::Q + qb * 8192, &p.tq, bar, qb * 64, c.g, c.t0, c.b);
    umma::tma_load_4d(st + S::KK + qb * 16384, &p.tk, bar, qb * 64, c.g, c.t0, c.b);
    umma::tma_load_4d(st + S::KK + qb * 16384 + 8192, &p.tkp, bar, qb * 64, c.g, c.t0 - p.shift, c.b);
  }
  umma::tma_load_4d(st + S::XX, &p.tx, bar, 0, c.h, c.t0, c.b);
  umma::tma_load_4d(st + S::XX + 8192, &p.txp, bar, 0, c.h, c.t0 - p.shift, c.b);
  umma::tma_load_4d(st + S::DY, &p.tdy, bar, 0, c.h, c.t0, c.b);
  umma::bulk_load(st + S::SIN, reinterpret_cast<const unsigned char*>(p.states) + (c.bh * p.nc + c.j) * (int64_t)NS * 128,
                  NS * 128, bar);
}

// token s of a chunk: adt, gamma, beta -> dst[s], dst[64 + s], dst[128 + s] (asynchronous copies)
__device__ __forceinline__ void bwd_prefetch_scalars(const TcBwdParams& p, const BwdChunk& c, int s, float* dst) {
  const int t = c.t0 + s;
  umma::cp_async4(dst + s, p.adt + (c.b * p.asb + t * p.ast + c.h * p.ash));
  umma::cp_async4(dst + 64 + s, p.gamma + (c.b * p.gsb + t * p.gst + c.h * p.gsh));
  umma::cp_async4(dst + 128 + s, p.beta + (c.b * p.bsb + t * p.bst + c.h * p.bsh));
  umma::cp_async_commit();
}

// The per-token scalars of a finished chunk (64 threads, s = 0-63 per thread, named barrier 1):
// dgamma, dbeta and dadt_u = sum_{t >= u} dc_t from the chunk's reductions in shared memory.
// sc: the chunk's [c | ec | w | wg wb | g | b]; wsel: which of the two warps this is.
__device__ __forceinline__ void bwd_token_tail(const TcBwdParams& p, const float* sc, const float* s_da, const float* s_xu,
                                               const float* s_pre, const float* s_dcint, float* s_tmp, int s, int lane,
                                               int wsel, float a_chunk, int b, int h, int t0) {
  const float* s_w = sc + 128;
  const float* s_g = sc + 320;
  const float* s_b = sc + 384;
  float da = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) da += s_da[i];
  float xu = 0.f, xpu = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    xu += s_xu[q * 128 + s];
    xpu += s_xu[q * 128 + 64 + s];
  }
  const float w = s_w[s];
  const float dw = s_g[s] * xu + s_b[s] * xpu;
  const float dg = s_pre[64 + s] + w * xu;
  const float db = s_pre[128 + s] + w * xpu;
  float dc = s_pre[s] + s_dcint[s] + s_dcint[64 + s] - w * dw;
  // dc_{L-1} += e^{c_L} da + sum_s w_s dw_s   (two warps: combine through shared memory)
  const float wdw = warp_sum(w * dw);
  if (lane == 0) s_tmp[wsel] = wdw;
  asm volatile("bar.sync 1, 64;" ::: "memory");
  if (s == 63) dc += a_chunk * da + s_tmp[0] + s_tmp[1];
  // dadt_u = sum_{t >= u} dc_t  (reverse cumulative sum over 64 tokens in two warps)
  const float total = warp_sum(dc);
  const float incl = warp_incl_scan(dc, lane);
  float suffix = total - incl + dc;
  if (lane == 0 && wsel == 1) s_tmp[2] = total;
  asm volatile("bar.sync 1, 64;" ::: "memory");
  if (wsel == 0) suffix += s_tmp[2];
  const int tt = t0 + s;
  p.dadt[b * p.dasb + (int64_t)tt * p.dast + h * p.dash] = suffix;
  p.dgamma[b * p.dgsb + (int64_t)tt * p.dgst + h * p.dgsh] = dg;
  p.dbeta[b * p.dbsb + (int64_t)tt * p.dbst + h * p.dbsh] = db;
}

template <int NS>
__global__ void __launch_bounds__(kBwdThreads, 1) ssd_bwd_tc_kernel(const __grid_constant__ TcBwdParams p) {
  using S = BwdSmem<NS>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sW = sm + S::W;
  unsigned char* sDYE = sW;  // e^{c_t} dY
  unsigned char* sPS = sW;   // [A | Ap]   [2][64 t][64 s]
  unsigned char* sXW = sW;   // [wgX | wbXp] (128 rows)
  unsigned char* sEG = sm + S::E;  // [Eg | Epb] [2][64 t][64 s]
  // Gn [NS n][64 p] goes over the current stage's S_in tile (set per chunk below)
  float* s_scal = reinterpret_cast<float*>(sm + S::SCAL);  // [2 parity][c | ec | w | wg wb | g | b]
  float* s_nx = s_scal + 2 * kScal;                            // next chunk's [adt | gamma | beta]
  float* s_rowZ = reinterpret_cast<float*>(sm + S::RED);  // [2 column block][2 half][64]
  float* s_colZ = s_rowZ + 256;                           // [4][128]
  float* s_colE = s_colZ + 512;                           // [4][128]
  float* s_xu = s_colE + 512;                             // [4][128]
  float* s_dcint = s_xu + 512;                            // [2][64]
  float* s_da = s_dcint + 128;                            // [16]
  float* s_tmp = s_da + 16;                               // [8]
  float* s_pre = s_tmp + 8;                               // [rowZ - colZ | colE g | colE b] per token
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BAR);
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + S::MISC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool scal_warp = (warp == 2 || warp == 3);  // stage and prepare the next chunk's scalars
  const int64_t total = p.B * p.H * p.nc;
  if (tid == 0) {
    misc[1] = atomicAdd(p.ticket, 1u);
    for (int i = 0; i < 5; ++i) umma::mbar_init(&bars[i], 1);
    umma::mbar_init(&bars[5], 8);  // the eight hand-off warps' writes of a chunk's state gradient
    umma::mbar_init(&bars[6], 8);  // the eight score-epilogue warps' tiles for the second group
    umma::mbar_fence_init();
  }
  __syncwarp();  // lane 0 of warp 0 rejoins before the warp-collective allocation
  if (warp == 0) {
    umma::tmem_alloc(&misc[0], 512);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = misc[0];
  const uint32_t R0 = tmem, R1 = tmem + 128, R2 = tmem + 256, R3 = tmem + 320, R4 = tmem + 384;
  uint32_t cur = misc[1];
  if (cur < total) {
    if (tid == 0) bwd_issue_loads<NS>(p, sm, &bars[0], bwd_chunk(p, cur));
    if (scal_warp) {
      bwd_prefetch_scalars(p, bwd_chunk(p, cur), tid - 64, s_nx);
      umma::cp_async_wait_all();
      chunk_scalars(s_scal, s_nx, tid - 64, lane);
    }
  }

  // the previous chunk's per-token scalars, written during this chunk's first MMA group
  bool pend = false;
  int pend_b = 0, pend_h = 0, pend_t0 = 0;
  uint32_t pend_par = 0;
  float pend_a = 0.f;
  const bool tail_warp = warp >= 14;
  for (uint32_t it = 0; cur < total; ++it) {
    const int stage = it & 1;
    const uint32_t par = it & 1;  // parity of this chunk's MMA-group barriers
    unsigned char* sQ = sm + stage * S::STAGE + S::Q;
    unsigned char* sKK = sm + stage * S::STAGE + S::KK;
    unsigned char* sXX = sm + stage * S::STAGE + S::XX;
    unsigned char* sDY = sm + stage * S::STAGE + S::DY;
    unsigned char* sSin = sm + stage * S::STAGE + S::SIN;
    unsigned char* sGN = sSin;  // Gn [NS n][64 p] replaces S_in once the first group is done
    const BwdChunk ck = bwd_chunk(p, cur);
    const int j = ck.j, b = ck.b, h = ck.h, g = ck.g, t0 = ck.t0;
    const int64_t bh = ck.bh;
    int* flags = p.flags + bh * (p.nc + 1);
    // Thread 32 is the producer: it takes the next ticket now, and while thread 0 waits for the
    // hand-off it drains the previous chunk's output tiles (its own TMA stores) and loads the next
    // chunk's operands into the other stage.
    uint32_t nx = 0, nxt = 0;
    bool prefetched = false, published = false;
    if (tid == 32) nx = atomicAdd(p.ticket, 1u);
    if (tid == 0) misc[2] = 0;  // failures of this chunk: bit 0 predecessor, 1 publish wait, 2 second group not issued
    // this chunk's scalars were prepared by the end of the previous one (or before the loop)
    const float* s_c = s_scal + (it & 1) * kScal;
    const float* s_ec = s_c + 64;
    const float* s_wgb = s_c + 192;  // [wg (64) | wb (64)]
    const float* s_g = s_c + 320;
    const float* s_b = s_c + 384;
    const bool load_ok = umma::mbar_wait(&bars[stage], (it >> 1) & 1, p.status);
    bool ok = __syncthreads_and(load_ok);
    const float a_chunk = expf(s_c[63]);

    if (ok) {
      // the products that need no rescaled operand start right away
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t q0 = umma::smem_u32(sQ), kk0 = umma::smem_u32(sKK), xx0 = umma::smem_u32(sXX);
        const uint32_t dy0 = umma::smem_u32(sDY), sin0 = umma::smem_u32(sSin);
        // b: S = Q [K;Kp]^T
        constexpr uint32_t idb = umma::idesc_bf16(64, 128, false, false);
#pragma unroll
        for (int ks = 0; ks < NS / 16; ++ks) {
          const uint32_t qb = ks >> 2, kin = ks & 3;
          umma::mma_bf16(R0, umma::desc_sw128(q0 + qb * 8192 + kin * 32, 16, 1024),
                         umma::desc_sw128(kk0 + qb * 16384 + kin * 32, 16, 1024), idb, ks > 0);
        }
        // a: dA = dY [X;Xp]^T
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma::mma_bf16(R0 + (16u << 16), umma::desc_sw128(dy0 + ks * 32, 16, 1024),
                         umma::desc_sw128(xx0 + ks * 32, 16, 1024), idb, ks > 0);
        // h: Ye = Q S_in^T
        constexpr uint32_t idh = umma::idesc_bf16(64, 64, false, true);
#pragma unroll
        for (int ks = 0; ks < NS / 16; ++ks) {
          const uint32_t qb = ks >> 2, kin = ks & 3;
          umma::mma_bf16(R1 + (16u << 16), umma::desc_sw128(q0 + qb * 8192 + kin * 32, 16, 1024),
                         umma::desc_sw128(sin0 + ks * 2048, 8192, 1024), idh, ks > 0);
        }
      }
      scale_rows(sDY, sDYE, 8192, s_ec, tid);   // e^{c_t} dY
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t q0 = umma::smem_u32(sQ);
        const uint32_t dye0 = umma::smem_u32(sDYE), sin0 = umma::smem_u32(sSin);
        // g: dSl' = Q^T dYe   (M = n)
        constexpr uint32_t idg = umma::idesc_bf16(NS, 64, true, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma::mma_bf16(R4, umma::desc_sw128(q0 + ks * 2048, 8192, 1024), umma::desc_sw128(dye0 + ks * 2048, 8192, 1024),
                         idg, ks > 0);
        // d (inter part): dQ = dYe S_in
        constexpr uint32_t idd1 = umma::idesc_bf16(64, NS, false, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma::mma_bf16(R1, umma::desc_sw128(dye0 + ks * 32, 16, 1024), umma::desc_sw128(sin0 + ks * 32, 16, 1024), idd1,
                         ks > 0);
        umma::mma_commit(&bars[2]);
      }
      if (pend && tail_warp)
        bwd_token_tail(p, s_scal + pend_par * kScal, s_da, s_xu, s_pre, s_dcint, s_tmp, tid - 448, lane, warp - 14, pend_a,
                       pend_b, pend_h, pend_t0);
      pend = false;
      if (tid == 32) misc[3] = nx;  // the next ticket, read by every thread after the barrier below
      ok = __syncthreads_and(umma::mbar_wait(&bars[2], par, p.status));
    }
    if (ok) {
      umma::fence_after_sync();
      published = true;  // warp 8 releases this chunk's flag below: ready, or aborted if the hand-off failed
      nxt = misc[3];
      if (scal_warp && nxt < total) bwd_prefetch_scalars(p, bwd_chunk(p, nxt), tid - 64, s_nx);  // next chunk
      if (warp < 8) {
        // score-gradient epilogue, warps 0-7.  Warp w: sub-partition sp = w % 4 (rows t = 16 sp +
        // lane % 16), half = w / 4 (0: K part with gamma, 1: Kp part with beta); it takes the two
        // 32-column blocks cc = 0, 1 in turn.  TMEM gives lanes 0-15 the S row and lanes 16-31 the
        // dA row; one swap per column pair hands lanes 0-15 columns 0-15 and lanes 16-31 columns
        // 16-31 of the block, so every lane works.
        const int sp = warp & 3, half = warp >> 2;
        const int t = 16 * sp + (lane & 15);
        const bool hiL = lane >= 16;
        const float* coef = half ? s_b : s_g;
        const float ct = s_c[t];
        const float* s_es = s_c + kScalEs;
        const bool fastm = s_c[kScalFast] != 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          float rowZ = 0.f;
          // decay e^{c_t - c_s}: this lane's 16 columns are two 8-token blocks, factorised when the
          // chunk allows it (chunk_scalars)
          const int r0 = cc * 32 + (hiL ? 16 : 0);
          const float et0 = fastm ? __expf(ct - s_c[r0]) : 0.f, et1 = fastm ? __expf(ct - s_c[r0 + 8]) : 0.f;
          auto epilogue = [&](auto decay) {
            float v[32];
            umma::tmem_ld32(R0 + ((uint32_t)(32 * sp) << 16) + half * 64 + cc * 32, v);
            float zc[16], ecs[16];
            uint32_t wa[8], we[8];
            float pa = 0.f, pe = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float recv = __shfl_xor_sync(0xffffffffu, hiL ? v[i] : v[16 + i], 16);
              const float sv = hiL ? recv : v[i];          // S_ts
              const float dav = hiL ? v[16 + i] : recv;    // dA_ts
              const int s = cc * 32 + (hiL ? 16 : 0) + i;
              const float m = (s <= t) ? decay(i, s) : 0.f;
              const float cf = coef[s];
              const float A = sv * cf * m;
              const float E = dav * m;
              const float z = dav * A;
              rowZ += z;
              zc[i] = z;
              ecs[i] = E * sv;
              const float eg = E * cf;
              if (i & 1) {
                wa[i >> 1] = pack_bf16(pa, A);
                we[i >> 1] = pack_bf16(pe, eg);
              } else {
                pa = A;
                pe = eg;
              }
            }
            // column sums over the 16 rows of this half-warp; lane keeps column (lane % 16)
            const float cz = colsum16(zc, lane), ce = colsum16(ecs, lane);
            const int col = half * 64 + cc * 32 + (hiL ? 16 : 0) + (lane & 15);
            s_colZ[sp * 128 + col] = cz;
            s_colE[sp * 128 + col] = ce;
            const int c0 = cc * 4 + (hiL ? 2 : 0);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              *reinterpret_cast<uint4*>(sPS + half * 8192 + umma::sw128_offset(t, c0 + q)) =
                  make_uint4(wa[4 * q], wa[4 * q + 1], wa[4 * q + 2], wa[4 * q + 3]);
              *reinterpret_cast<uint4*>(sEG + half * 8192 + umma::sw128_offset(t, c0 + q)) =
                  make_uint4(we[4 * q], we[4 * q + 1], we[4 * q + 2], we[4 * q + 3]);
            }
          };
          if (fastm)
            epilogue([&](int i, int s) { return (i < 8 ? et0 : et1) * s_es[s]; });
          else
            epilogue([&](int, int s) { return __expf(ct - s_c[s]); });
          rowZ += __shfl_xor_sync(0xffffffffu, rowZ, 16);
          if (lane < 16) s_rowZ[(cc * 2 + half) * 64 + t] = rowZ;
        }
        // The second group needs only these tiles: thread 0 issues it once the eight epilogue warps
        // are done (their arrivals on bars[6] follow the proxy fence for [A | Ap], [Eg | Epb] and the
        // TMEM fence for the loads of R0, which the group overwrites), while the hand-off goes on.
        umma::fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(&bars[6]);
        if (tid == 0) {
          if (umma::mbar_wait(&bars[6], par, p.status)) {
            umma::fence_after_sync();
            const uint32_t q0 = umma::smem_u32(sQ), kk0 = umma::smem_u32(sKK), dy0 = umma::smem_u32(sDY);
            const uint32_t ps0 = umma::smem_u32(sPS), eg0 = umma::smem_u32(sEG);
            // c: dXc = [A|Ap]^T dY   (M = s|s')
            constexpr uint32_t idc = umma::idesc_bf16(128, 64, true, true);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma::mma_bf16(R2, umma::desc_sw128(ps0 + ks * 2048, 8192, 1024), umma::desc_sw128(dy0 + ks * 2048, 8192, 1024),
                             idc, ks > 0);
            // d (intra part): dQ += [Eg|Epb] [K;Kp]
            constexpr uint32_t idd2 = umma::idesc_bf16(64, NS, false, true);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t part = ks >> 2, kin = ks & 3;
              umma::mma_bf16(R1, umma::desc_sw128(eg0 + part * 8192 + kin * 32, 16, 1024),
                             umma::desc_sw128(kk0 + part * 8192 + kin * 2048, 16384, 1024), idd2, 1);
            }
            // e: dK = [Eg|Epb]^T Q   (M = s|s')
            constexpr uint32_t ide = umma::idesc_bf16(128, NS, true, true);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma::mma_bf16(R0, umma::desc_sw128(eg0 + ks * 2048, 8192, 1024), umma::desc_sw128(q0 + ks * 2048, 8192, 1024),
                             ide, ks > 0);
            umma::mma_commit(&bars[3]);
          } else {
            atomicOr(&misc[2], 4u);  // the second group was not issued
          }
        }
      } else {
        // reverse state hand-off, warps 8-15, beside the score epilogue (it needs only the first
        // group's dSl' and the neighbour's state):  G[j] = dSl'^T + e^{c_L} G[j+1];
        // da = <G[j+1], S_in[j]>.  Warp w: sub-partition sp = w % 4 (state rows n), p-quarters
        // pq = (w - 8) / 4 and pq + 2 (16 columns each).
        const int hw = warp - 8, sp = warp & 3;
        const bool rows128 = (NS == 128);
        const int n = rows128 ? 32 * sp + lane : 16 * sp + (lane & 15);
        const bool active = rows128 || lane < 16;
        int fl = kFlagReady;
        if (lane == 0 && j != p.nc - 1) fl = wait_flag(&flags[j + 1], p.status);
        fl = __shfl_sync(0xffffffffu, fl, 0);
        float da_part = 0.f;
        if (fl == kFlagReady) {
          // ring slots are [p/4][n][4]; the caller's dfinal / dinitial states are [p][n]
          const int64_t PN = (int64_t)kP * NS;
          float* dinit = (j == 0 && p.dinit) ? p.dinit + bh * PN : nullptr;
#pragma unroll 1
          for (int k = 0; k < 2; ++k) {
            const int pq = (hw >> 2) + 2 * k;
            float ds[16], gn[16];
            umma::tmem_ld16(R4 + ((uint32_t)(32 * sp) << 16) + 16 * pq, ds);
            if (active) {
              if (j == p.nc - 1) {
#pragma unroll
                for (int i = 0; i < 16; ++i) gn[i] = p.dfin ? __ldcg(p.dfin + bh * PN + (16 * pq + i) * NS + n) : 0.f;
              } else {
                const float4* s4 =
                    reinterpret_cast<const float4*>(p.ring + (bh * 2 + ((j + 1) & 1)) * PN) + 4 * pq * NS + n;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float4 v = __ldcg(s4 + q * NS);
                  gn[4 * q] = v.x; gn[4 * q + 1] = v.y; gn[4 * q + 2] = v.z; gn[4 * q + 3] = v.w;
                }
              }
              float4* d4 = reinterpret_cast<float4*>(p.ring + (bh * 2 + (j & 1)) * PN) + 4 * pq * NS + n;
#pragma unroll
              for (int q = 0; q < 4; ++q)
                d4[q * NS] = make_float4(ds[4 * q] + a_chunk * gn[4 * q], ds[4 * q + 1] + a_chunk * gn[4 * q + 1],
                                         ds[4 * q + 2] + a_chunk * gn[4 * q + 2], ds[4 * q + 3] + a_chunk * gn[4 * q + 3]);
              if (dinit) {
#pragma unroll
                for (int i = 0; i < 16; ++i) dinit[(16 * pq + i) * NS + n] = ds[i] + a_chunk * gn[i];
              }
              // Gn (bf16, [n][p] like S_in) replaces S_in in its tile: the first group, the only
              // reader of S_in, is done; each thread reads the S_in chunk it then overwrites
#pragma unroll
              for (int qd = 0; qd < 2; ++qd) {
                float sv[8];
                load_chunk(sSin, n, 2 * pq + qd, sv);
#pragma unroll
                for (int e = 0; e < 8; ++e) da_part += gn[8 * qd + e] * sv[e];
                *reinterpret_cast<uint4*>(sGN + umma::sw128_offset(n, 2 * pq + qd)) =
                    make_uint4(pack_bf16(gn[8 * qd], gn[8 * qd + 1]), pack_bf16(gn[8 * qd + 2], gn[8 * qd + 3]),
                               pack_bf16(gn[8 * qd + 4], gn[8 * qd + 5]), pack_bf16(gn[8 * qd + 6], gn[8 * qd + 7]));
              }
            }
          }
        } else if (lane == 0) {
          atomicOr(&misc[2], 1u);
        }
        // Publish G[j] once every hand-off warp has written its part: each warp's arrival on
        // bars[5] (release) follows its writes, warp 8 waits for all eight (acquire) and releases
        // the flag, which is cumulative over what it has observed.  The wait is bounded.
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(&bars[5]);
        if (warp == 8) {
          const bool all = umma::mbar_wait(&bars[5], par, p.status);
          if (lane == 0) {
            if (!all) atomicOr(&misc[2], 2u);
            st_release(&flags[j], misc[2] == 0 ? kFlagReady : kFlagAbort);
          }
        }
        da_part = warp_sum(da_part);
        if (lane == 0) s_da[hw] = da_part;
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      const uint32_t fails = misc[2];
      ok = fails == 0;
      // thread 32 (the producer) drains the previous chunk's output tiles (its own TMA stores) and
      // loads the next chunk's operands into the other stage while the second group runs
      if (tid == 32) {
        umma::bulk_wait_read();
        if (nx < total) {
          bwd_issue_loads<NS>(p, sm + (stage ^ 1) * S::STAGE, &bars[stage ^ 1], bwd_chunk(p, nx));
          prefetched = true;
        }
      }
      // [wgX | wbXp] takes the place of [A | Ap] once the second group has read it; an issued group
      // is also waited for on the way out after a failed hand-off (TMEM is freed at exit)
      bool g2 = false;
      if (!(fails & 4u)) {
        g2 = umma::mbar_wait(&bars[3], par, p.status);
        if (ok && g2) scale_rows(sXX, sXW, 16384, s_wgb, tid);
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      ok = __syncthreads_and(ok && g2);
    }
    if (ok) {
      if (tid == 0) {
        umma::fence_after_sync();
        const uint32_t kk0 = umma::smem_u32(sKK), xw0 = umma::smem_u32(sXW), gn0 = umma::smem_u32(sGN);
        // e (state part): dK += [wgX;wbXp] Gn
        constexpr uint32_t ide2 = umma::idesc_bf16(128, NS, false, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma::mma_bf16(R0, umma::desc_sw128(xw0 + ks * 32, 16, 1024), umma::desc_sw128(gn0 + ks * 32, 16, 1024), ide2, 1);
        // f: U = [K;Kp] Gn^T
        constexpr uint32_t idf = umma::idesc_bf16(128, 64, false, true);
#pragma unroll
        for (int ks = 0; ks < NS / 16; ++ks) {
          const uint32_t qb = ks >> 2, kin = ks & 3;
          umma::mma_bf16(R3, umma::desc_sw128(kk0 + qb * 16384 + kin * 32, 16, 1024),
                         umma::desc_sw128(gn0 + ks * 2048, 8192, 1024), idf, ks > 0);
        }
        umma::mma_commit(&bars[4]);
      }
      // While the third group runs: dQ (final since the second group) leaves TMEM for the dq staging
      // tile over Q (dead now), with the dc inter term from Ye (R1 lanes +16); warps 2-3 reduce the
      // per-token sums of the score epilogue.
      {
        __syncwarp();  // lane 0 rejoins warp 0 before the warp-collective TMEM load
        umma::fence_after_sync();
        const int sp = warp & 3, cq = warp >> 2;
        if (32 * cq < NS) {
          const int t = 16 * sp + (lane & 15);
          float v[32];
          umma::tmem_ld32(R1 + ((uint32_t)(32 * sp) << 16) + 32 * cq, v);
          if (lane < 16) stage_row32(sQ + (cq >> 1) * 8192, t, 4 * (cq & 1), v);
          if (lane >= 16 && cq < 2) {
            float acc = 0.f;
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              float d[8];
              load_chunk(sDY, t, 4 * cq + qd, d);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc += d[e] * v[8 * qd + e];
            }
            s_dcint[cq * 64 + t] = s_ec[t] * acc;
          }
        }
        if (scal_warp) {
          const int s = tid - 64;
          float colZ = 0.f, colEg = 0.f, colEb = 0.f, rowZ = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            colZ += s_colZ[q * 128 + s] + s_colZ[q * 128 + 64 + s];
            colEg += s_colE[q * 128 + s];
            colEb += s_colE[q * 128 + 64 + s];
            rowZ += s_rowZ[q * 64 + s];
          }
          s_pre[s] = rowZ - colZ;
          s_pre[64 + s] = colEg;
          s_pre[128 + s] = colEb;
          if (nxt < total) {  // the next chunk's scalars (its other-parity block is free)
            umma::cp_async_wait_all();  // this thread's own copies
            chunk_scalars(s_scal + ((it + 1) & 1) * kScal, s_nx, tid - 64, lane);
          }
        }
      }
      ok = __syncthreads_and(umma::mbar_wait(&bars[4], par, p.status));
    } else if (tid == 0 && !published) {
      st_release(&flags[j], kFlagAbort);
    }
    if (ok) {
      umma::fence_after_sync();
      // warp w: sub-partition sp = w % 4, column quarter cq = w / 4
      const int sp = warp & 3, cq = warp >> 2;
      // Output tiles are staged (bf16, 128-byte swizzle) in shared memory that is dead by now and
      // leave through TMA stores: dq -> Q tile (staged while the third group ran), dk | dkp -> K/Kp
      // tiles, dx | dxp -> X/Xp tiles (each thread overwrites exactly the X elements it has just read).
      unsigned char* st_dq = sQ;
      unsigned char* st_dk = sKK;
      unsigned char* st_dkp = sKK + S::QB * 8192;
      unsigned char* st_dx = sXX;
      unsigned char* st_dxp = sXX + 8192;
      // (2) dx / dxp rows: dXc (R2) + w g U (R3), columns [16 cq, 16 cq + 16); x.U partial sums for
      // dgamma / dbeta
      {
        const int r = 32 * sp + lane;  // 0-63: s of X, 64-127: s of Xp
        float dxc[16], u[16];
        umma::tmem_ld16x2(R2 + ((uint32_t)(32 * sp) << 16) + 16 * cq, R3 + ((uint32_t)(32 * sp) << 16) + 16 * cq, dxc, u);
        const float wgt = s_wgb[r];  // wg for X rows, wb for Xp rows
        float xu = 0.f;
#pragma unroll
        for (int qd = 0; qd < 2; ++qd) {
          float xv[8];
          load_chunk(sXX, r, 2 * cq + qd, xv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            xu += xv[e] * u[8 * qd + e];
            dxc[8 * qd + e] += wgt * u[8 * qd + e];
          }
        }
        s_xu[cq * 128 + r] = xu;
        stage_row16(r < 64 ? st_dx : st_dxp, r & 63, 2 * cq, dxc);
      }
      // (3) dk / dkp rows (R0), columns [32 cq, 32 cq + 32)
      if (32 * cq < NS) {
        const int r = 32 * sp + lane;
        float v[32];
        umma::tmem_ld32(R0 + ((uint32_t)(32 * sp) << 16) + 32 * cq, v);
        stage_row32((r < 64 ? st_dk : st_dkp) + (cq >> 1) * 8192, r & 63, 4 * (cq & 1), v);
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 32) {  // the producer waits for these before reusing the stage
#pragma unroll
        for (int qb = 0; qb < S::QB; ++qb) {
          umma::tma_store_4d(&p.tdq, st_dq + qb * 8192, qb * 64, g, t0, b);
          umma::tma_store_4d(&p.tdk, st_dk + qb * 8192, qb * 64, g, t0, b);
          umma::tma_store_4d(&p.tdkp, st_dkp + qb * 8192, qb * 64, g, t0, b);
        }
        umma::tma_store_4d(&p.tdx, st_dx, 0, h, t0, b);
        umma::tma_store_4d(&p.tdxp, st_dxp, 0, h, t0, b);
        umma::bulk_commit();
      }
      // this chunk's per-token scalars are written by warps 14-15 while the next chunk's first MMA
      // group runs (or after the loop)
      pend = true;
      pend_b = b;
      pend_h = h;
      pend_t0 = t0;
      pend_par = it & 1;
      pend_a = a_chunk;
    }
    __syncthreads();  // every read of this stage and of the work tiles is done
    if (!ok) {
      // leave after an error; the ticket already taken is aborted and its loads land first
      if (tid == 32 && nx < total) {
        const BwdChunk cn = bwd_chunk(p, nx);
        st_release(&p.flags[cn.bh * (p.nc + 1) + cn.j], kFlagAbort);
        if (prefetched) umma::mbar_wait(&bars[stage ^ 1], ((it + 1) >> 1) & 1, p.status);
      }
      break;
    }
    cur = nxt;
  }
  if (pend && tail_warp)  // the last chunk's per-token scalars
    bwd_token_tail(p, s_scal + pend_par * kScal, s_da, s_xu, s_pre, s_dcint, s_tmp, tid - 448, lane, warp - 14, pend_a,
                   pend_b, pend_h, pend_t0);
  if (tid == 32) umma::bulk_wait_all();  // staged output tiles must be read out before exit
  if (scal_warp) umma::cp_async_wait_all();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------------------
// state-only passes (context parallelism, segmented long sequences): no per-token outputs.
//   forward : S_in[j+1] = e^{c_L} S_in[j] + [K;Kp]^T [wgX; wbXp]   (MMA M=N, N=64, K=128)
//   backward: G[j] = Q^T (e^{c} dY) + e^{c_L} G[j+1]                 (MMA M=N, N=64, K=64)
// 128 threads, 64 TMEM columns, <= 65 KB shared memory: several CTAs per SM hide the hand-off.

constexpr int kStThreads = 128;

template <int NS>
struct StateSmem {
  static constexpr int QB = NS / 64;
  static constexpr uint32_t A0 = 0;                    // fwd: [QB][K | Kp]   bwd: Q [QB][64][64]
  static constexpr uint32_t B0 = A0 + QB * 16384;      // fwd: [X | Xp]       bwd: dY
  static constexpr uint32_t B1 = B0 + 16384;           // fwd: [wgX | wbXp]   bwd: e^c dY
  static constexpr uint32_t SCAL = B1 + 16384;         // c, w*g, w*b (or e^c) : 3 x 64 floats
  static constexpr uint32_t BAR = SCAL + 3 * 256;
  static constexpr uint32_t MISC = BAR + 2 * 8;
  static constexpr uint32_t TOTAL = MISC + 16;
  static constexpr uint32_t ALLOC = TOTAL + 1024;
};

struct TcStateParams {
  CUtensorMap t0, t1, t2, t3;  // fwd: k, kp, x, xp   bwd: q, dy
  int64_t B, T, H, G;
  int nc;
  const float* adt;
  const float* gamma;
  const float* beta;
  int64_t asb, ast, ash, gsb, gst, gsh, bsb, bst, bsh;
  const float* init;   // fwd: initial state [B*H][P][N] or null;  bwd: dfinal or null
  float* out;          // fwd: final state;  bwd: dinitial state (both [B*H][P][N], may be null)
  float* ring;         // [B*H][2] slots, [p/4][n][4]
  unsigned int* ticket;
  int* flags;
  int32_t* status;
  int shift;           // as in TcFwdParams (t1 / t3 of the forward read one token earlier)
};

template <int NS, bool BACKWARD>
__global__ void __launch_bounds__(kStThreads) ssd_state_tc_kernel(const __grid_constant__ TcStateParams p) {
  using S = StateSmem<NS>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = sm + S::A0;
  unsigned char* sB0 = sm + S::B0;
  unsigned char* sB1 = sm + S::B1;
  float* s_c = reinterpret_cast<float*>(sm + S::SCAL);
  float* s_f0 = s_c + 64;   // fwd: w*g   bwd: e^{c}
  float* s_f1 = s_c + 128;  // fwd: w*b
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BAR);
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + S::MISC);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    misc[1] = atomicAdd(p.ticket, 1u);
    umma::mbar_init(&bars[0], 1);
    umma::mbar_init(&bars[1], 1);
    umma::mbar_fence_init();
  }
  __syncwarp();  // lane 0 of warp 0 rejoins before the warp-collective allocation
  if (warp == 0) {
    umma::tmem_alloc(&misc[0], 64);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = misc[0];
  const UnitIdx u = decode_ticket(misc[1], p.B, p.H, p.G);
  const int j = BACKWARD ? p.nc - 1 - u.chunk : u.chunk;
  const int64_t bh = u.bh;
  const int b = u.b, h = u.h, g = u.g;
  const int t0 = j * kL;
  int* flags = p.flags + bh * (p.nc + 1);
  const int64_t PN = (int64_t)kP * NS;

  if (tid == 0) {
    if (BACKWARD) {
      umma::mbar_arrive_expect_tx(&bars[0], S::QB * 8192 + 8192);
#pragma unroll
      for (int qb = 0; qb < S::QB; ++qb) umma::tma_load_4d(sA + qb * 8192, &p.t0, &bars[0], qb * 64, g, t0, b);
      umma::tma_load_4d(sB0, &p.t1, &bars[0], 0, h, t0, b);
    } else {
      umma::mbar_arrive_expect_tx(&bars[0], S::QB * 16384 + 16384);
#pragma unroll
      for (int qb = 0; qb < S::QB; ++qb) {
        umma::tma_load_4d(sA + qb * 16384, &p.t0, &bars[0], qb * 64, g, t0, b);
        umma::tma_load_4d(sA + qb * 16384 + 8192, &p.t1, &bars[0], qb * 64, g, t0 - p.shift, b);
      }
      umma::tma_load_4d(sB0, &p.t2, &bars[0], 0, h, t0, b);
      umma::tma_load_4d(sB0 + 8192, &p.t3, &bars[0], 0, h, t0 - p.shift, b);
    }
  }
  if (tid < 64) {
    const int t = t0 + tid;
    const float a = p.adt[b * p.asb + t * p.ast + h * p.ash];
    if (!BACKWARD) {
      s_f0[tid] = p.gamma[b * p.gsb + t * p.gst + h * p.gsh];
      s_f1[tid] = p.beta[b * p.bsb + t * p.bst + h * p.bsh];
    }
    s_c[tid] = warp_incl_scan(a, lane);
  }
  __syncthreads();
  if (tid >= 32 && tid < 64) s_c[tid] += s_c[31];
  __syncthreads();
  if (tid < 64) {
    const float c = s_c[tid];
    if (BACKWARD) {
      s_f0[tid] = expf(c);
    } else {
      const float w = expf(s_c[63] - c);
      s_f0[tid] *= w;
      s_f1[tid] *= w;
    }
  }
  const bool load_ok = umma::mbar_wait(&bars[0], 0, p.status);
  __syncthreads();
  const float a_chunk = expf(s_c[63]);
  bool ok = __syncthreads_and(load_ok);
  if (ok) {
    // rescale the rows of the x (fwd) or dy (bwd) tile(s) into B1
    const uint32_t bytes = BACKWARD ? 8192u : 16384u;
    for (uint32_t off = (uint32_t)tid * 16u; off < bytes; off += kStThreads * 16u) {
      const int r = off >> 7;
      const float f = BACKWARD ? s_f0[r] : (r < 64 ? s_f0[r] : s_f1[r - 64]);
      const uint4 v = *reinterpret_cast<const uint4*>(sB0 + off);
      uint4 o;
      float2 e;
      e = unpack_bf16(v.x); o.x = pack_bf16(e.x * f, e.y * f);
      e = unpack_bf16(v.y); o.y = pack_bf16(e.x * f, e.y * f);
      e = unpack_bf16(v.z); o.z = pack_bf16(e.x * f, e.y * f);
      e = unpack_bf16(v.w); o.w = pack_bf16(e.x * f, e.y * f);
      *reinterpret_cast<uint4*>(sB1 + off) = o;
    }
    umma::fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      umma::fence_after_sync();
      const uint32_t a0 = umma::smem_u32(sA), b1 = umma::smem_u32(sB1);
      constexpr uint32_t id = umma::idesc_bf16(NS, 64, true, true);
      if (BACKWARD) {
        // G_loc^T[n][p] = sum_t q_t[n] e^{c_t} dy_t[p]   (A = Q^T, B = e^c dY, both MN-major)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma::mma_bf16(tmem, umma::desc_sw128(a0 + ks * 2048, 8192, 1024), umma::desc_sw128(b1 + ks * 2048, 8192, 1024),
                         id, ks > 0);
      } else {
        // S_loc^T[n][p] = sum_s k_s[n] wg_s x_s[p] + kp_s[n] wb_s xp_s[p]
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t part = ks >> 2, kin = ks & 3;
          umma::mma_bf16(tmem, umma::desc_sw128(a0 + part * 8192 + kin * 2048, 16384, 1024),
                         umma::desc_sw128(b1 + part * 8192 + kin * 2048, 8192, 1024), id, ks > 0);
        }
      }
      umma::mma_commit(&bars[1]);
    }
    ok = __syncthreads_and(umma::mbar_wait(&bars[1], 0, p.status));
  }
  if (ok) {
    umma::fence_after_sync();
    // this thread's n (lane of the MMA's D layout) and all 64 p
    const int sp = warp;
    const bool rows128 = (NS == 128);
    const int n = rows128 ? 32 * sp + lane : 16 * sp + (lane & 15);
    const bool active = rows128 || lane < 16;
    float v0[32], v1[32];
    umma::tmem_ld32x2(tmem + ((uint32_t)(32 * sp) << 16), tmem + ((uint32_t)(32 * sp) << 16) + 32, v0, v1);
    if (tid == 0) {
      const bool first = BACKWARD ? (j == p.nc - 1) : (j == 0);
      misc[2] = first ? kFlagReady : wait_flag(&flags[BACKWARD ? j + 1 : j], p.status);
    }
    __syncthreads();
    ok = misc[2] == kFlagReady;
    if (ok && active) {
      const bool first = BACKWARD ? (j == p.nc - 1) : (j == 0);
      const bool last = BACKWARD ? (j == 0) : (j == p.nc - 1);
      const int in_slot = BACKWARD ? ((j + 1) & 1) : (j & 1);
      const int out_slot = BACKWARD ? (j & 1) : ((j + 1) & 1);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const float* loc = half ? v1 : v0;
        float prev[32];
        if (first) {
#pragma unroll
          for (int i = 0; i < 32; ++i) prev[i] = p.init ? __ldcg(p.init + bh * PN + (32 * half + i) * NS + n) : 0.f;
        } else {
          const float4* s4 = reinterpret_cast<const float4*>(p.ring + (bh * 2 + in_slot) * PN) + 8 * half * NS + n;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v = __ldcg(s4 + q * NS);
            prev[4 * q] = v.x; prev[4 * q + 1] = v.y; prev[4 * q + 2] = v.z; prev[4 * q + 3] = v.w;
          }
        }
        float4* d4 = reinterpret_cast<float4*>(p.ring + (bh * 2 + out_slot) * PN) + 8 * half * NS + n;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          d4[q * NS] = make_float4(a_chunk * prev[4 * q] + loc[4 * q], a_chunk * prev[4 * q + 1] + loc[4 * q + 1],
                                   a_chunk * prev[4 * q + 2] + loc[4 * q + 2], a_chunk * prev[4 * q + 3] + loc[4 * q + 3]);
        if (last && p.out) {
#pragma unroll
          for (int i = 0; i < 32; ++i) p.out[bh * PN + (32 * half + i) * NS + n] = a_chunk * prev[i] + loc[i];
        }
      }
    }
    // the barrier orders every thread's ring writes before thread 0's release (cumulative)
    __syncthreads();
    if (tid == 0) st_release(&flags[BACKWARD ? j : j + 1], ok ? kFlagReady : kFlagAbort);
  } else if (tid == 0) {
    st_release(&flags[BACKWARD ? j : j + 1], kFlagAbort);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------------------------
// host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D map over a [B, T, H(or G), D] bf16 view: dims (D, H, T, B), box (64, 1, 64, 1), 128-byte swizzle
bool make_map(CUtensorMap* map, const zb_view& v, int64_t B, int64_t T, int64_t H, int64_t D) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)v.sh * 2, (cuuint64_t)v.st * 2, (cuuint64_t)v.sb * 2};
  const cuuint32_t box[4] = {64, 1, 64, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v.ptr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// TMA needs a 16-byte aligned base and positive strides that are multiples of 16 bytes.
bool view_tma_ok(const zb_view& v) {
  const auto a16 = [](int64_t x) { return x > 0 && (x * 2) % 16 == 0 && x * 2 < (1ll << 40); };
  return v.ptr && reinterpret_cast<uintptr_t>(v.ptr) % 16 == 0 && a16(v.sh) && a16(v.st) && a16(v.sb);
}

// streaming multiprocessors of the current device (cached per device)
int sm_count() {
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

constexpr int64_t kRingBandBytes = 32ll << 20;

template <int NS>
int launch_fwd(const zb_ssd_args* a, ChainSync sync, void* states, void* ring, cudaStream_t stream) {
  TcFwdParams p;
  memset(&p, 0, sizeof(p));
  if (!make_map(&p.tq, a->q, a->B, a->T, a->G, NS) || !make_map(&p.tk, a->k, a->B, a->T, a->G, NS) ||
      !make_map(&p.tkp, a->kp, a->B, a->T, a->G, NS) || !make_map(&p.tx, a->x, a->B, a->T, a->H, kP) ||
      !make_map(&p.txp, a->xp, a->B, a->T, a->H, kP) || !make_map(&p.ty, a->y, a->B, a->T, a->H, kP))
    return ZB_ERR_LAYOUT;
  p.B = a->B; p.T = a->T; p.H = a->H; p.G = a->G;
  p.nc = (int)(a->T / kL);
  p.adt = static_cast<const float*>(a->adt.ptr);
  p.gamma = static_cast<const float*>(a->gamma.ptr);
  p.beta = static_cast<const float*>(a->beta.ptr);
  p.asb = a->adt.sb; p.ast = a->adt.st; p.ash = a->adt.sh;
  p.gsb = a->gamma.sb; p.gst = a->gamma.st; p.gsh = a->gamma.sh;
  p.bsb = a->beta.sb; p.bst = a->beta.st; p.bsh = a->beta.sh;
  p.y = static_cast<__nv_bfloat16*>(a->y.ptr);
  p.ysb = a->y.sb; p.yst = a->y.st; p.ysh = a->y.sh;
  p.init = static_cast<const float*>(a->initial_state);
  p.fin = static_cast<float*>(a->final_state);
  p.states = static_cast<__nv_bfloat16*>(states);
  p.ring = static_cast<float*>(ring);
  p.ticket = sync.ticket;
  p.flags = sync.flags;
  p.status = a->status;
  p.shift = (a->flags & ZB_FLAG_SHIFTED) ? 1 : 0;
  auto k = ssd_fwd_tc_kernel<NS>;
  const int smem = (int)FwdSmem<NS>::ALLOC;
  if (dyn_smem(reinterpret_cast<const void*>(k), smem) != ZB_OK) return ZB_ERR_CUDA;
  // persistent: CTAS_PER_SM CTAs per SM
  const int64_t units = a->B * a->H * p.nc, slots = (int64_t)FwdSmem<NS>::CTAS_PER_SM * sm_count();
  // A chain's ring slot is read back one row of its band's chunks after it is written; with all chains
  // in one chunk-major order (B64 x H32 at N = 64: 64 MB of slots) the slots leave L2 in between and
  // cost DRAM traffic.  Bands of at most kRingBandBytes of slots (and at least one chain per CTA)
  // keep them resident.
  const int64_t ring_chain = 2LL * kP * NS * (int64_t)sizeof(float);
  const int64_t band = std::max<int64_t>(kRingBandBytes / ring_chain, slots);
  p.band = (uint32_t)std::min<int64_t>(a->B * a->H, band);
  const dim3 grid((unsigned)(units < slots ? units : slots));
  k<<<grid, FwdSmem<NS>::THREADS, smem, stream>>>(p);
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}


template <int NS>
int launch_bwd(const zb_ssd_args* a, ChainSync sync, void* ring, cudaStream_t stream) {
  TcBwdParams p;
  memset(&p, 0, sizeof(p));
  if (!view_tma_ok(a->dy)) return ZB_ERR_LAYOUT;
  const zb_view* outs[] = {&a->dx, &a->dxp, &a->dq, &a->dk, &a->dkp};
  for (auto v : outs)
    if (!view_tma_ok(*v)) return ZB_ERR_LAYOUT;
  if (!make_map(&p.tdq, a->dq, a->B, a->T, a->G, NS) || !make_map(&p.tdk, a->dk, a->B, a->T, a->G, NS) ||
      !make_map(&p.tdkp, a->dkp, a->B, a->T, a->G, NS) || !make_map(&p.tdx, a->dx, a->B, a->T, a->H, kP) ||
      !make_map(&p.tdxp, a->dxp, a->B, a->T, a->H, kP))
    return ZB_ERR_LAYOUT;
  if (!make_map(&p.tq, a->q, a->B, a->T, a->G, NS) || !make_map(&p.tk, a->k, a->B, a->T, a->G, NS) ||
      !make_map(&p.tkp, a->kp, a->B, a->T, a->G, NS) || !make_map(&p.tx, a->x, a->B, a->T, a->H, kP) ||
      !make_map(&p.txp, a->xp, a->B, a->T, a->H, kP) || !make_map(&p.tdy, a->dy, a->B, a->T, a->H, kP))
    return ZB_ERR_LAYOUT;
  p.B = a->B; p.T = a->T; p.H = a->H; p.G = a->G;
  p.nc = (int)(a->T / kL);
  p.adt = static_cast<const float*>(a->adt.ptr);
  p.gamma = static_cast<const float*>(a->gamma.ptr);
  p.beta = static_cast<const float*>(a->beta.ptr);
  p.asb = a->adt.sb; p.ast = a->adt.st; p.ash = a->adt.sh;
  p.gsb = a->gamma.sb; p.gst = a->gamma.st; p.gsh = a->gamma.sh;
  p.bsb = a->beta.sb; p.bst = a->beta.st; p.bsh = a->beta.sh;
  p.states = static_cast<const __nv_bfloat16*>(a->states);
  p.dfin = static_cast<const float*>(a->dfinal_state);
  p.dinit = static_cast<float*>(a->dinitial_state);
  p.ring = static_cast<float*>(ring);
  p.dx = static_cast<__nv_bfloat16*>(a->dx.ptr); p.dxsb = a->dx.sb; p.dxst = a->dx.st; p.dxsh = a->dx.sh;
  p.dxp = static_cast<__nv_bfloat16*>(a->dxp.ptr); p.dxpsb = a->dxp.sb; p.dxpst = a->dxp.st; p.dxpsh = a->dxp.sh;
  p.dq = static_cast<__nv_bfloat16*>(a->dq.ptr); p.dqsb = a->dq.sb; p.dqst = a->dq.st; p.dqsh = a->dq.sh;
  p.dk = static_cast<__nv_bfloat16*>(a->dk.ptr); p.dksb = a->dk.sb; p.dkst = a->dk.st; p.dksh = a->dk.sh;
  p.dkp = static_cast<__nv_bfloat16*>(a->dkp.ptr); p.dkpsb = a->dkp.sb; p.dkpst = a->dkp.st; p.dkpsh = a->dkp.sh;
  p.dadt = static_cast<float*>(a->dadt.ptr); p.dasb = a->dadt.sb; p.dast = a->dadt.st; p.dash = a->dadt.sh;
  p.dgamma = static_cast<float*>(a->dgamma.ptr); p.dgsb = a->dgamma.sb; p.dgst = a->dgamma.st; p.dgsh = a->dgamma.sh;
  p.dbeta = static_cast<float*>(a->dbeta.ptr); p.dbsb = a->dbeta.sb; p.dbst = a->dbeta.st; p.dbsh = a->dbeta.sh;
  p.ticket = sync.ticket;
  p.flags = sync.flags;
  p.status = a->status;
  p.shift = (a->flags & ZB_FLAG_SHIFTED) ? 1 : 0;
  auto k = ssd_bwd_tc_kernel<NS>;
  const int smem = (int)BwdSmem<NS>::ALLOC;
  if (dyn_smem(reinterpret_cast<const void*>(k), smem) != ZB_OK) return ZB_ERR_CUDA;
  const int64_t units = a->B * a->H * p.nc;
  const dim3 grid((unsigned)(units < sm_count() ? units : sm_count()));  // persistent: one CTA per SM
  k<<<grid, kBwdThreads, smem, stream>>>(p);
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}

template <int NS, bool BACKWARD>
int launch_state(const zb_ssd_args* a, ChainSync sync, void* ring, cudaStream_t stream) {
  TcStateParams p;
  memset(&p, 0, sizeof(p));
  bool maps_ok;
  if (BACKWARD) {
    maps_ok = view_tma_ok(a->dy) && make_map(&p.t0, a->q, a->B, a->T, a->G, NS) &&
              make_map(&p.t1, a->dy, a->B, a->T, a->H, kP);
  } else {
    maps_ok = make_map(&p.t0, a->k, a->B, a->T, a->G, NS) && make_map(&p.t1, a->kp, a->B, a->T, a->G, NS) &&
              make_map(&p.t2, a->x, a->B, a->T, a->H, kP) && make_map(&p.t3, a->xp, a->B, a->T, a->H, kP);
  }
  if (!maps_ok) return ZB_ERR_LAYOUT;
  p.B = a->B; p.T = a->T; p.H = a->H; p.G = a->G;
  p.nc = (int)(a->T / kL);
  p.adt = static_cast<const float*>(a->adt.ptr);
  p.gamma = static_cast<const float*>(a->gamma.ptr);
  p.beta = static_cast<const float*>(a->beta.ptr);
  p.asb = a->adt.sb; p.ast = a->adt.st; p.ash = a->adt.sh;
  p.gsb = a->gamma.sb; p.gst = a->gamma.st; p.gsh = a->gamma.sh;
  p.bsb = a->beta.sb; p.bst = a->beta.st; p.bsh = a->beta.sh;
  p.init = static_cast<const float*>(BACKWARD ? a->dfinal_state : a->initial_state);
  p.out = static_cast<float*>(BACKWARD ? a->dinitial_state : a->final_state);
  p.ring = static_cast<float*>(ring);
  p.ticket = sync.ticket;
  p.flags = sync.flags;
  p.status = a->status;
  p.shift = (a->flags & ZB_FLAG_SHIFTED) ? 1 : 0;
  auto k = ssd_state_tc_kernel<NS, BACKWARD>;
  const int smem = (int)StateSmem<NS>::ALLOC;
  if (dyn_smem(reinterpret_cast<const void*>(k), smem) != ZB_OK) return ZB_ERR_CUDA;
  k<<<(unsigned)(a->B * a->H * p.nc), kStThreads, smem, stream>>>(p);
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}

}  // namespace

bool tc_supported(const zb_ssd_args* a) {
  if (a->dtype != ZB_BF16 || a->scalar_dtype != ZB_F32) return false;
  if (a->P != kP || (a->N != 64 && a->N != 128)) return false;
  if (a->T % kL != 0) return false;
  if (a->T / kL >= (1 << 30) || a->B * a->H * (a->T / kL) >= (1ll << 31)) return false;
  const zb_view* v[] = {&a->x, &a->q, &a->k, &a->kp, &a->xp};
  for (auto x : v)
    if (!view_tma_ok(*x)) return false;
  if (a->y.ptr && (reinterpret_cast<uintptr_t>(a->y.ptr) % 16 || (a->y.sh * 2) % 16 || (a->y.st * 2) % 16 ||
                   (a->y.sb * 2) % 16))
    return false;
  return encode_fn() != nullptr;
}

// The tensor-core backward handles one q/k group per head (G == H, the reference's layout);
// grouped q/k (G < H) differentiate on the SIMT path.
bool tc_has_backward(const zb_ssd_args* a) { return a->G == a->H; }

int tc_chunk() { return kL; }

size_t tc_states_bytes(const zb_ssd_args* a) {
  return align_up((size_t)a->B * a->H * (a->T / kL) * a->N * kP * 2, 256);
}

// forward and backward both need the two-slot fp32 hand-off ring per (batch, head)
size_t tc_workspace_bytes(const zb_ssd_args* a, bool) {
  return align_up((size_t)a->B * a->H * 2 * kP * a->N * sizeof(float), 256);
}

int tc_fwd(const zb_ssd_args* a, ChainSync sync, void* states, void* ws, cudaStream_t stream) {
  if (a->flags & ZB_FLAG_STATE_ONLY) {
    if (a->N == 128) return launch_state<128, false>(a, sync, ws, stream);
    if (a->N == 64) return launch_state<64, false>(a, sync, ws, stream);
    return ZB_ERR_UNSUPPORTED;
  }
  if (a->N == 128) return launch_fwd<128>(a, sync, states, ws, stream);
  if (a->N == 64) return launch_fwd<64>(a, sync, states, ws, stream);
  return ZB_ERR_UNSUPPORTED;
}

int tc_bwd(const zb_ssd_args* a, ChainSync sync, void* ws, cudaStream_t stream) {
  if (a->flags & ZB_FLAG_STATE_ONLY) {
    if (a->N == 128) return launch_state<128, true>(a, sync, ws, stream);
    if (a->N == 64) return launch_state<64, true>(a, sync, ws, stream);
    return ZB_ERR_UNSUPPORTED;
  }
  if (a->G != a->H) return ZB_ERR_UNSUPPORTED;
  if (a->N == 128) return launch_bwd<128>(a, sync, ws, stream);
  if (a->N == 64) return launch_bwd<64>(a, sync, ws, stream);
  return ZB_ERR_UNSUPPORTED;
}

}  // namespace zb
