// ska_common.cuh -- shared definitions of the SKA core kernels (sm_100a).
//
// Data model (one (batch b, head h) "series" of T tokens, split into
// C = ceil(T / CS) chunks of CS tokens; the tail chunk is zero padded as in
// KLF/koopman_lm/ska.py:87-94):
//
//   raw chunk statistics of chunk c (unnormalised keys z, values v):
//     G'_c = sum_{t in c} z_t z_t^T                          r x r
//     M'_c = sum_{t in c} z_{t+1} z_t^T                      r x r
//            (the transition that leaves chunk c is owned by chunk c, which
//             folds the reference's boundary term ska.py:108-111,125-129
//             into the ordinary exclusive scan)
//     C'_c = sum_{t in c} v_t z_t^T                          P x r
//   exclusive (decayed) scan over chunks:  X_excl[c] = a * X_excl[c-1] + X'[c-1]
//   (a = 1 for the standard strategy, ska.py:114-133; a = decay_alpha for the
//    decay strategy, adaptive_chunking.py:225-238).
//
//   The shared key norm m = max_t ||z_t|| (ska.py:441) enters only as scalars:
//   Gn = G_excl / m^2 + ridge I,  Mn = M_excl / m^2,  Cn = C_excl / m,
//   Qn = zq / m.  Raw statistics are therefore computed once and scaled.
//
//   Per chunk operator (L = chol(Gn), Li = L^{-1}, S = Li^T Li = Gn^{-1}):
//     A0 = Mn S,  A = clamp(gamma,1,1.5) / max(sigma(A0),1) * A0
//     W  = Cn Li^T A^K Li                                    P x r
//     y_t = W qn_t  for t in chunk c
//   which equals B_v L A^K L^{-1} qn of ska.py:165-181.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace ska {

constexpr int kMaxRank = 64;
constexpr int kMaxP = 128;
constexpr int kMaxChunk = 256;
constexpr int kMaxPowerK = 8;
constexpr int kThreads = 256;
constexpr int kPowerIters = 6;        // ska.py:41 (n_iters=6)
constexpr float kJitter = 1e-4f;      // ska.py:142
constexpr float kNormClamp = 1e-6f;   // ska.py:441
constexpr float kPowerEps = 1e-8f;    // ska.py:53,55

struct Dims {
  int B, T, H, r, P, CS, C, K;
  int decay;        // 0: standard, 1: decay
  float ridge;
  float alpha;      // 1 for standard
  int SW;           // floats per statistics record: 2 r r + P r
  uint32_t wlim;    // polls before a tensor-core kernel's first wait of a role gives up
};

struct In {
  const void* p;
  long long sb, st, sh;
};
struct Out {
  void* p;
  long long sb, st, sh;
};

template <typename T>
__device__ __forceinline__ float load_elem(const T* p);
template <>
__device__ __forceinline__ float load_elem<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// value -> float for an element already held in registers (no memory access)
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ void store_elem(T* p, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

template <typename T>
__device__ __forceinline__ float ld_tok(const In& x, int b, int t, int h, int j) {
  const T* base = static_cast<const T*>(x.p);
  return load_elem<T>(base + (long long)b * x.sb + (long long)t * x.st + (long long)h * x.sh + j);
}
template <typename T>
__device__ __forceinline__ void st_tok(const Out& x, int b, int t, int h, int j, float v) {
  T* base = static_cast<T*>(x.p);
  store_elem<T>(base + (long long)b * x.sb + (long long)t * x.st + (long long)h * x.sh + j, v);
}

// ---- saved (forward -> backward) and scratch layouts -----------------------

__host__ __device__ constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Chunk operators kept by the bf16 forward for the backward.  r <= 32: one 32 x 32
// fp32 row-major tile each (rows and columns past r hold the padding the warp
// kernels use: identity for Li and S, zero elsewhere, identity for A^K when K = 0):
constexpr int kOpLi = 0, kOpA = 1, kOpAK = 2, kOpU = 3, kOpV = 4, kOpS = 5, kNumOps = 6;
constexpr int kOpFloats = 32 * 32;
// 32 < r <= 64: one 64 x 64 matrix each, as the four-warp kernels hold it in shared
// memory (four swizzled 32 x 32 tiles, column-block major), in the order Li, S,
// A0 = Mn S (unscaled), A0^K (unscaled), U, V
constexpr int kQOpLi = 0, kQOpS = 1, kQOpA0 = 2, kQOpA0K = 3, kQOpU = 4, kQOpV = 5;
constexpr int kQOpFloats = 64 * 64;

// (the four-warp kernels take r % 8 == 0 and P <= 64)
__host__ __device__ constexpr size_t ops_floats_per_chunk(long long r, long long P) {
  return r <= 32 ? (size_t)kNumOps * kOpFloats
                 : (r <= 64 && r % 8 == 0 && P <= 64) ? (size_t)kNumOps * kQOpFloats : 0;
}

struct SavedLayout {
  size_t stats;     // float [B][H][C][SW]  exclusive-scanned raw statistics
  size_t cmax;      // u64   [B][H][C]      packed (norm bits, ~t) chunk maxima
  size_t invs;      // float [B][H][C]      1 / max(sigma, 1)
  size_t flags;     // int   [B][H][C]      bit0: jittered, bit1: jitter failed too
  size_t status;    // int   [B][H][C]      tensor-core statistics kernel: 0 ok,
                    //                      1 TMA wait expired, 2 MMA wait expired
  size_t wm;        // bf16 hi, lo planes [B][H][C][2][r/8][P][8]: W / m as the
                    //   tensor-core operand of the readout products
  size_t lis;       // the factor kernels' Li, for the operator kernels: r <= 32,
                    //   float [B][H][C][32][32] (Li^T, kept-operator layout); 32 < r <= 64,
                    //   float [B][H][C][3][32][32] (Li's non-zero 32 x 32 tiles)
  size_t fwd;       // bytes a forward needs when no backward reads its buffer
  size_t ops;       // float [B][H][C][ops_floats_per_chunk(r, P)]: Li = L^{-1}, A, A^K,
                    //   U = A^K Li, V = Li^T U, S = Li^T Li, written by bf16 forwards
                    //   given the whole buffer (total bytes) and read by the backward
  size_t total;
};

struct ScratchLayout {
  size_t dstats;    // float [B][H][C][SW]  gradients of the raw statistics
  size_t dmpart;    // float [B][H][C]      per-chunk partial d(max norm)
  size_t dgpart;    // float [B][H][C]      per-chunk partial d(gamma)
  size_t dm;        // float [B][H]
  size_t status;    // int   [B][H][C]      tensor-core backward kernels: bits 0-1 the
                    //                      readout-gradient kernel, bits 2-3 the token
                    //                      kernel; each 0 ok, 1 copy wait expired,
                    //                      2 product wait expired
  size_t dw;        // float [B][H][C][P r] raw readout gradient sum_t dy_t zq_t^T
  size_t total;
};

__host__ __device__ inline SavedLayout saved_layout(long long B, long long H, long long C, long long SW,
                                                   long long r, long long P) {
  SavedLayout L{};
  const size_t n = (size_t)B * H * C;
  size_t off = 0;
  L.stats = off; off = align256(off + n * SW * sizeof(float));
  L.cmax = off;  off = align256(off + n * sizeof(unsigned long long));
  L.invs = off;  off = align256(off + n * sizeof(float));
  L.flags = off; off = align256(off + n * sizeof(int));
  L.status = off; off = align256(off + n * sizeof(int));
  L.wm = off;    off = align256(off + (r <= 64 ? n * (size_t)P * r * 4 : 0));
  L.lis = off;
  off = align256(off + (r <= 32 ? n * (size_t)1024 * 4 : ops_floats_per_chunk(r, P) ? n * (size_t)3 * 1024 * 4 : 0));
  L.fwd = off;
  L.ops = off;   off = align256(off + n * ops_floats_per_chunk(r, P) * sizeof(float));
  L.total = off;
  return L;
}

__host__ __device__ inline ScratchLayout scratch_layout(long long B, long long H, long long C, long long SW,
                                                       long long r, long long P) {
  ScratchLayout L{};
  const size_t n = (size_t)B * H * C;
  size_t off = 0;
  L.dstats = off; off = align256(off + n * SW * sizeof(float));
  L.dmpart = off; off = align256(off + n * sizeof(float));
  L.dgpart = off; off = align256(off + n * sizeof(float));
  L.dm = off;     off = align256(off + (size_t)B * H * sizeof(float));
  L.status = off; off = align256(off + n * sizeof(int));
  L.dw = off;     off = align256(off + n * (size_t)P * r * sizeof(float));
  L.total = off;
  return L;
}

// x = hi + lo as bf16 pairs (round to nearest twice): 8 floats -> two 16-byte rows
__device__ __forceinline__ void split_bf16x8(const float (&x)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
    const float2 hf = __bfloat1622float2(hh);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(x[2 * e] - hf.x, x[2 * e + 1] - hf.y);
    h[e] = *reinterpret_cast<const uint32_t*>(&hh);
    l[e] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Packed arg-max key: larger norm wins, ties go to the smaller token index
// (the first maximum, as torch.max(dim) / numpy.argmax return on the CPU).
__device__ __forceinline__ unsigned long long pack_max(float norm, int t) {
  return ((unsigned long long)__float_as_uint(norm) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (unsigned)t);
}
__device__ __forceinline__ float unpack_norm(unsigned long long k) {
  return __uint_as_float((unsigned)(k >> 32));
}
__device__ __forceinline__ int unpack_t(unsigned long long k) {
  return (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull));
}

// Caller-provided timing events (ska_set_profile_events); nullptr = off.
struct ProfileEvents {
  cudaEvent_t ev[10];
  bool on;
};
ProfileEvents* profile_events();
inline void prof_record(int i, cudaStream_t st) {
  ProfileEvents* p = profile_events();
  if (p->on) cudaEventRecord(p->ev[i], st);
}

}  // namespace ska
