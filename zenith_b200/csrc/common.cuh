// Shared device helpers for the SSD kernels: dtype I/O, strided views and the chained
// (ticket-ordered) state hand-off between the CTAs that own consecutive chunks.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "zb_ssd.h"

namespace zb {

// ---------------------------------------------------------------------------------------------
// element conversion
template <typename T> struct Conv;
template <> struct Conv<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ double to_d(float v) { return v; }
  static __device__ __forceinline__ float from_d(double v) { return (float)v; }
};
template <> struct Conv<double> {
  static __device__ __forceinline__ float to_f(double v) { return (float)v; }
  static __device__ __forceinline__ double from_f(float v) { return v; }
  static __device__ __forceinline__ double to_d(double v) { return v; }
  static __device__ __forceinline__ double from_d(double v) { return v; }
};
template <> struct Conv<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ double to_d(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_d(double v) { return __float2bfloat16_rn((float)v); }
};
template <> struct Conv<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ double to_d(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_d(double v) { return __float2half_rn((float)v); }
};

// load an element of type T as accumulator type TA / store TA as T
template <typename TA, typename T> __device__ __forceinline__ TA ldv(const T* p) {
  if constexpr (sizeof(TA) == 8) return Conv<T>::to_d(*p); else return Conv<T>::to_f(*p);
}
template <typename TA, typename T> __device__ __forceinline__ void stv(T* p, TA v) {
  if constexpr (sizeof(TA) == 8) *p = Conv<T>::from_d(v); else *p = Conv<T>::from_f(v);
}

template <typename TA> __device__ __forceinline__ TA xexp(TA v);
template <> __device__ __forceinline__ float xexp<float>(float v) { return expf(v); }
template <> __device__ __forceinline__ double xexp<double>(double v) { return exp(v); }

// eight consecutive elements (16-byte aligned) as 16-byte accesses
template <typename T> struct Vec8;
template <> struct Vec8<float> {
  static __device__ __forceinline__ void ld(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void st(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
};
template <> struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
// eight consecutive elements held packed in registers (bf16: one 16-byte word)
template <typename T> struct Pack8;
template <> struct Pack8<__nv_bfloat16> {
  uint4 u;
  __device__ __forceinline__ void ld(const __nv_bfloat16* p) { u = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ float get(int e) const {
    const uint32_t w = e < 2 ? u.x : e < 4 ? u.y : e < 6 ? u.z : u.w;
    return __uint_as_float((e & 1) ? (w & 0xffff0000u) : (w << 16));
  }
};
template <> struct Pack8<float> {
  float4 a, b;
  __device__ __forceinline__ void ld(const float* p) {
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
  }
  __device__ __forceinline__ float get(int e) const {
    const float4& q = e < 4 ? a : b;
    const int k = e & 3;
    return k == 0 ? q.x : k == 1 ? q.y : k == 2 ? q.z : q.w;
  }
};

// A [B, T, H, D] view with element strides; the innermost dimension is contiguous.
struct View {
  const void* ptr;
  int64_t sb, st, sh;
  template <typename T> __device__ __forceinline__ const T* row(int64_t b, int64_t t, int64_t h) const {
    return reinterpret_cast<const T*>(ptr) + b * sb + t * st + h * sh;
  }
  template <typename T> __device__ __forceinline__ T* wrow(int64_t b, int64_t t, int64_t h) const {
    return const_cast<T*>(reinterpret_cast<const T*>(ptr)) + b * sb + t * st + h * sh;
  }
};

// ---------------------------------------------------------------------------------------------
// chained hand-off
//
// CTAs take a ticket from a global counter when they start, and the ticket (not blockIdx)
// decides which chunk they own.  Tickets are handed out in chunk order, so the owner of the
// chunk a CTA waits for started earlier and is resident: every wait ends.  Waits are still
// bounded (about one second): on expiry the CTA records ZB_ERR_TIMEOUT in the status word,
// marks its own hand-off as aborted (flag value 2) so that its successors stop at once, and
// returns.

constexpr int kFlagReady = 1;
constexpr int kFlagAbort = 2;
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s
constexpr uint32_t kWaitMaxIters = 1u << 22;         // independent cap: seconds at one L2 load per poll

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int32_t* p) { return *(volatile const int32_t*)p; }

// Called by one thread. Returns kFlagReady, or kFlagAbort on an aborted predecessor / timeout.
static __device__ __noinline__ int wait_flag(const int* flag, int32_t* status) {
  const uint64_t t0 = globaltimer();
  uint32_t sleep_ns = 32;
  for (uint32_t it = 0; it < kWaitMaxIters; ++it) {
    const int v = ld_acquire(flag);
    if (v == kFlagReady) return kFlagReady;
    if (v != 0) return kFlagAbort;
    if ((it & 15) == 15) {
      if (ld_volatile(status) != 0) return kFlagAbort;
      if (globaltimer() - t0 > kWaitTimeoutNs) break;
    }
    __nanosleep(sleep_ns);
    if (sleep_ns < 64) sleep_ns <<= 1;
  }
  atomicCAS(status, 0, (int32_t)ZB_ERR_TIMEOUT);
  return kFlagAbort;
}

// Scratch layout shared by all chained kernels: [ticket counter | pad to 256 | flags[n_flags]].
struct ChainSync {
  unsigned int* ticket;
  int* flags;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The (batch, head, chunk) unit of ticket tk, tickets in chunk-major order:
// tk = chunk * (B*H) + b * H + h.  32-bit arithmetic (64-bit division is a long software
// routine); the argument checks bound B*H*T below 2^31.
struct UnitIdx {
  int chunk, b, h, g;
  uint32_t bh;
};
__device__ __forceinline__ UnitIdx decode_ticket(uint32_t tk, int64_t B, int64_t H, int64_t G) {
  const uint32_t h32 = (uint32_t)H, bh32 = (uint32_t)B * h32;
  UnitIdx u;
  const uint32_t c = tk / bh32;
  u.chunk = (int)c;
  u.bh = tk - c * bh32;
  const uint32_t b = u.bh / h32;
  u.b = (int)b;
  u.h = (int)(u.bh - b * h32);
  u.g = (int)((uint32_t)u.h / (h32 / (uint32_t)G));
  return u;
}
// Banded order: the chains are taken `band` at a time (the last band may hold fewer), each band in
// chunk-major order: tk = start * nc + chunk * size + (bh - start) for the band [start, start + size).
// A chain's chunk j still has a lower ticket than its chunk j + 1, so the argument above holds, and
// only one band's ring slots are live at a time.  band >= B*H gives the chunk-major order.
__device__ __forceinline__ UnitIdx decode_ticket_banded(uint32_t tk, int64_t B, int64_t H, int64_t G, int nc,
                                                        uint32_t band) {
  const uint32_t h32 = (uint32_t)H, bh32 = (uint32_t)B * h32;
  const uint32_t per_band = band * (uint32_t)nc;
  const uint32_t bi = tk / per_band;
  const uint32_t start = bi * band;
  const uint32_t size = min(band, bh32 - start);
  const uint32_t r = tk - bi * per_band;
  const uint32_t c = r / size;
  UnitIdx u;
  u.chunk = (int)c;
  u.bh = start + (r - c * size);
  const uint32_t b = u.bh / h32;
  u.b = (int)b;
  u.h = (int)(u.bh - b * h32);
  u.g = (int)((uint32_t)u.h / (h32 / (uint32_t)G));
  return u;
}
inline size_t chain_sync_bytes(int64_t n_flags) { return align_up(256 + (size_t)n_flags * sizeof(int), 256); }

// ---------------------------------------------------------------------------------------------
// warp helpers
template <typename TA> __device__ __forceinline__ TA warp_sum(TA v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <typename TA> __device__ __forceinline__ TA warp_incl_scan(TA v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    TA u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

}  // namespace zb
