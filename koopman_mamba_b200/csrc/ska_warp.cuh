// ska_warp.cuh -- register-resident warp primitives for the per-chunk SKA algebra
// (rank r <= 32).  One warp owns one chunk; lane i owns row i of every r x r
// matrix (rows past r are padding: identity for the Gram factor, zero elsewhere,
// which leaves every real entry unchanged).
//
// Shared-memory tiles are 32 x 32 fp32, row-major with a 16-byte-chunk XOR
// swizzle (chunk q of row k stored at chunk q ^ (k & 7)): a lane writing its
// own row with 128-bit stores and a warp reading one row as a broadcast are
// both conflict-free, and so is a warp reading one column.
#pragma once

#include "ska_common.cuh"

namespace ska {
namespace wpc {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float shfl(float v, int src) { return __shfl_sync(kFull, v, src); }

__device__ __forceinline__ int swz(int row, int col) {
  return row * 32 + ((((col >> 2) ^ (row & 7)) << 2) | (col & 3));
}

// this lane's 32-float register row -> row `row` of tile T
__device__ __forceinline__ void st_row(float* T, int row, const float (&v)[32]) {
  float4* p = reinterpret_cast<float4*>(T + row * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) p[q ^ (row & 7)] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
__device__ __forceinline__ void ld_row(float (&v)[32], const float* T, int row) {
  const float4* p = reinterpret_cast<const float4*>(T + row * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 x = p[q ^ (row & 7)];
    v[4 * q] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
}
// column `col` of tile T (K rows) -> v[0..K)
template <int K>
__device__ __forceinline__ void ld_col(float (&v)[K], const float* T, int col) {
#pragma unroll
  for (int k = 0; k < K; ++k) v[k] = T[swz(k, col)];
}
// this lane's register row written as COLUMN `col` of tile T (K rows)
template <int K>
__device__ __forceinline__ void st_col(float* T, int col, const float (&v)[K]) {
#pragma unroll
  for (int k = 0; k < K; ++k) T[swz(k, col)] = v[k];
}

// (d0, d1) += (a0, a1) * (b0, b1) as one packed fp32x2 FMA (sm_100)
__device__ __forceinline__ void fma2p(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  unsigned long long dd, bb, aa;
  float2 dv = make_float2(d0, d1), bv = make_float2(b0, b1), av = make_float2(a0, a1);
  dd = *reinterpret_cast<unsigned long long*>(&dv);
  bb = *reinterpret_cast<unsigned long long*>(&bv);
  aa = *reinterpret_cast<unsigned long long*>(&av);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(dd) : "l"(aa), "l"(bb));
  dv = *reinterpret_cast<float2*>(&dd);
  d0 = dv.x;
  d1 = dv.y;
}

__device__ __forceinline__ void fma2(float& d0, float& d1, float a, float b0, float b1) {
  unsigned long long dd, bb, aa;
  float2 dv = make_float2(d0, d1), bv = make_float2(b0, b1), av = make_float2(a, a);
  dd = *reinterpret_cast<unsigned long long*>(&dv);
  bb = *reinterpret_cast<unsigned long long*>(&bv);
  aa = *reinterpret_cast<unsigned long long*>(&av);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(dd) : "l"(aa), "l"(bb));
  dv = *reinterpret_cast<float2*>(&dd);
  d0 = dv.x;
  d1 = dv.y;
}

// Compiler-only fence: keeps fully unrolled loops from hoisting every shared-memory
// load ahead of the arithmetic (which would need ~1000 live registers).
__device__ __forceinline__ void sched_fence() { asm volatile("" ::: "memory"); }

// acc[j] += sum_{k<K} a[k] T[k][j]  (T: K rows of a swizzled 32-column tile, read as broadcasts)
template <int K>
__device__ __forceinline__ void mac_tile(float (&acc)[32], const float (&a)[K], const float* T) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if ((k & 1) == 0) sched_fence();
    const float4* row = reinterpret_cast<const float4*>(T + k * 32);
    const float ak = a[k];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = row[q ^ (k & 7)];
      fma2(acc[4 * q], acc[4 * q + 1], ak, b.x, b.y);
      fma2(acc[4 * q + 2], acc[4 * q + 3], ak, b.z, b.w);
    }
  }
}

// out[j] = sum_{k<32} a[k] T[j][k]  (a times T^T; T rows read as broadcasts)
__device__ __forceinline__ void dot_rows(float (&out)[32], const float (&a)[32], const float* T) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if ((j & 1) == 0) sched_fence();
    const float4* row = reinterpret_cast<const float4*>(T + j * 32);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = row[q ^ (j & 7)];
      fma2p(s0, s1, a[4 * q], a[4 * q + 1], b.x, b.y);
      fma2p(s0, s1, a[4 * q + 2], a[4 * q + 3], b.z, b.w);
    }
    out[j] = s0 + s1;
  }
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(kFull, x, o);
    x = y > x ? y : x;
  }
  return x;
}

template <int N>
__device__ __forceinline__ void zero(float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = 0.f;
}

__device__ __forceinline__ float warp_sum32(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

// In-place Cholesky of the 32 x 32 matrix whose row `lane` is g (lower part read),
// fused with the inverse of the factor.  On success g = row `lane` of L (zero upper
// part) and x = column `lane` of L^{-1}.  Returns false at the first non-positive
// pivot (uniform), like potrf's info > 0 (ska.py:140).
// Right-looking: at step j the warp broadcasts column j of L (L[k][j] from lane k);
// the same values drive the forward substitution L x = e_lane, so the inverse costs
// no extra shuffles.  1/L[j][j] comes from rsqrtf (a few ulp).
__device__ __forceinline__ bool chol_inv32(float (&g)[32], float (&x)[32], int lane) {
#pragma unroll
  for (int k = 0; k < 32; ++k) x[k] = (k == lane) ? 1.f : 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float djj = shfl(g[j], j);
    if (!(djj > 0.f)) return false;
    const float rs = rsqrtf(djj);                      // 1 / L[j][j]
    const float lij = lane > j ? g[j] * rs : (lane == j ? djj * rs : 0.f);
    g[j] = lij;
    x[j] *= rs;                                        // Li[j][lane] is final
#pragma unroll
    for (int k = j + 1; k < 32; ++k) {
      const float lkj = shfl(lij, k);                  // L[k][j]
      g[k] = fmaf(-lij, lkj, g[k]);
      x[k] = fmaf(-lkj, x[j], x[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < 32; ++k)
    if (k > lane) g[k] = 0.f;
  return true;
}

// chol_inv32 with the column broadcasts through 32 floats of the warp's shared
// memory (cb, 16-byte aligned) instead of shuffles: at step j each lane stores its
// entry of column j and every lane reads the whole column back as 8 broadcast
// loads, so that a step costs one store, eight loads and the FMAs (the shuffle
// version issues 31 - j shuffles per step, and twelve or more warps per SM doing
// that saturate the shuffle unit).  Same results and return value as chol_inv32,
// up to the rounding of the fused scale.  TRIM: the steps past n (warp-uniform) are
// skipped; rows and columns past n must hold the identity padding, which those
// steps would leave unchanged (a template switch, so that the full-size factor
// keeps its straight-line code: a run-time test in it, or a second trimmed copy
// beside it, slowed the r = 32 operator kernel by 2-11 us at B=8, H=12, L=2048).
template <bool TRIM = false>
__device__ __forceinline__ bool chol_inv32_bc(float (&g)[32], float (&x)[32], float* cb, int lane, int n = 32) {
#pragma unroll
  for (int k = 0; k < 32; ++k) x[k] = (k == lane) ? 1.f : 0.f;
  const float4* cb4 = reinterpret_cast<const float4*>(cb);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (TRIM && j >= n) break;
    cb[lane] = g[j];
    __syncwarp();
    float c[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 v = cb4[q];
      c[4 * q] = v.x;
      c[4 * q + 1] = v.y;
      c[4 * q + 2] = v.z;
      c[4 * q + 3] = v.w;
    }
    __syncwarp();
    const float djj = c[j];
    if (!(djj > 0.f)) return false;
    const float rs = rsqrtf(djj);                      // 1 / L[j][j]
    const float lij = lane > j ? g[j] * rs : (lane == j ? djj * rs : 0.f);
    g[j] = lij;
    x[j] *= rs;                                        // Li[j][lane] is final
    const float lr = lij * rs, xr = x[j] * rs;         // L[k][j] = c[k] rs
#pragma unroll
    for (int k = j + 1; k < 32; ++k) {
      g[k] = fmaf(-lr, c[k], g[k]);
      x[k] = fmaf(-xr, c[k], x[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < 32; ++k)
    if (k > lane) g[k] = 0.f;
  return true;
}

// one halving step of the butterfly reduce-scatter: keep half N of the live
// entries t[0..2N), exchange the other half with lane ^ OFF
template <int N, int OFF>
__device__ __forceinline__ void rs_step(float (&t)[32], int lane) {
  const bool up = (lane & OFF) != 0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float send = up ? t[i] : t[i + N];
    const float keep = up ? t[i + N] : t[i];
    t[i] = keep + __shfl_xor_sync(kFull, send, OFF);
  }
}
// out_lane = sum over lanes j of t_j[lane]  (butterfly reduce-scatter, 31 shuffles)
__device__ __forceinline__ float reduce_scatter32(float (&t)[32], int lane) {
  rs_step<16, 16>(t, lane);
  rs_step<8, 8>(t, lane);
  rs_step<4, 4>(t, lane);
  rs_step<2, 2>(t, lane);
  rs_step<1, 1>(t, lane);
  return t[0];
}

// sigma_max estimate of ska.py:41-58: 6 power iterations from v = 1/sqrt(r) on the
// matrix whose row `lane` is a (zero rows/cols past r).  x / max(||x||, 1e-8) is
// taken as x * min(rsqrt(||x||^2), 1e8).
__device__ __forceinline__ float power_sigma32(const float (&a)[32], int lane, int r) {
  float v = lane < r ? rsqrtf((float)r) : 0.f;
  float u = 0.f;
#pragma unroll 1
  for (int it = 0; it <= kPowerIters; ++it) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      s0 = fmaf(a[j], shfl(v, j), s0);
      s1 = fmaf(a[j + 1], shfl(v, j + 1), s1);
      s2 = fmaf(a[j + 2], shfl(v, j + 2), s2);
      s3 = fmaf(a[j + 3], shfl(v, j + 3), s3);
    }
    u = (s0 + s1) + (s2 + s3);
    if (it == kPowerIters) break;
    u *= fminf(rsqrtf(warp_sum32(u * u)), 1.f / kPowerEps);
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) t[i] = u * a[i];
    const float w = reduce_scatter32(t, lane);
    v = w * fminf(rsqrtf(warp_sum32(w * w)), 1.f / kPowerEps);
  }
  return sqrtf(warp_sum32(u * u));
}

// ---- tensor-core readout helpers (mma.sync m16n8k8 TF32) ----
// ---- per-chunk record access shared by the chunk kernels ----
__host__ __device__ inline int p_blocks(int P) { return (P + 31) >> 5; }

__device__ __forceinline__ void build_gram_row(float (&g)[32], const float (&grow)[32], const float (&gcol)[32],
                                               int lane, int r, float im2, float ridge, float jit) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float v;
    if (lane < r && j < r) {
      v = 0.5f * (grow[j] * im2 + gcol[j] * im2);   // ska.py:119,138
      if (j == lane) v += ridge + jit;
    } else {
      v = (j == lane) ? 1.f : 0.f;
    }
    g[j] = v;
  }
}

// Global loads are issued unconditionally from clamped (always valid) addresses and
// masked afterwards, so that a lane's loads are all in flight together.

// row `row` of the nrows x ncols row-major global matrix src, times `scale`, zero padded
__device__ __forceinline__ void ld_gmem_row(float (&v)[32], const float* src, int row, int nrows, int ncols,
                                            float scale) {
  const bool rv = row < nrows;
  const float* p = src + (size_t)(rv ? row : 0) * ncols;
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    float4 x[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) x[q] = __ldg(p4 + q);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[4 * q] = rv ? x[q].x * scale : 0.f;
      v[4 * q + 1] = rv ? x[q].y * scale : 0.f;
      v[4 * q + 2] = rv ? x[q].z * scale : 0.f;
      v[4 * q + 3] = rv ? x[q].w * scale : 0.f;
    }
  } else {
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __ldg(p + (j < ncols ? j : 0));
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (rv && j < ncols) ? x[j] * scale : 0.f;
  }
}

// Tile T <- rows [0, nrows) of a row-major nrows x ncols fp32 matrix in global
// memory, times scale (rows and columns past it zero).  With ncols == 32 and a
// 16-byte aligned source the warp reads 512 contiguous bytes per instruction
// (lane-per-row loads touch 32 cache lines per instruction instead).  Rows of T
// are written by other lanes: synchronise the warp before and after.
// Not inlined (one copy per translation unit): the chunk kernels stall on
// instruction fetch, and one shared copy of each record mover beats a copy per
// call site (backward 0.202 -> 0.1945 ms, forward 0.1009 -> 0.0969 ms at B=8,
// H=12, L=2048, P=64, r=32).
static __device__ __noinline__ void load_mat(float* T, const float* src, int nrows, int ncols, float scale, int lane) {
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int f = 32 * k + lane;
      v[k] = __ldg(s4 + ((f >> 3) < nrows ? f : 0));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int f = 32 * k + lane, row = f >> 3, q = f & 7;
      const bool ok = row < nrows;
      const float4 x = make_float4(ok ? v[k].x * scale : 0.f, ok ? v[k].y * scale : 0.f, ok ? v[k].z * scale : 0.f,
                                   ok ? v[k].w * scale : 0.f);
      reinterpret_cast<float4*>(T + row * 32)[q ^ (row & 7)] = x;
    }
  } else {
    float v[32];
    ld_gmem_row(v, src, lane, nrows, ncols, scale);
    st_row(T, lane, v);
  }
}

// rows [0, nrows) x columns [0, ncols) of a row-major global matrix -> tile T by
// asynchronous 16-byte copies (cp.async, L2 only); the rest of the tile is zeroed by
// zero-length sources.  Returns false, and copies nothing, unless ncols % 4 == 0
// and src is 16-byte aligned (then call load_mat instead).  The copies belong to
// the lane's next cp_async_commit group; wait for it and synchronise the warp
// before reading the tile.
__device__ __forceinline__ bool cp_tile_async(float* T, const float* src, int nrows, int ncols, int lane) {
  if ((ncols & 3) != 0 || (reinterpret_cast<uintptr_t>(src) & 15) != 0) return false;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int f = 32 * k + lane, row = f >> 3, q = f & 7;
    const bool ok = row < nrows && 4 * q < ncols;
    const float* s = src + (ok ? row * ncols + 4 * q : 0);
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(T + row * 32 + ((q ^ (row & 7)) << 2)));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(s), "r"(ok ? 16 : 0) : "memory");
  }
  return true;
}
// Kept chunk operators (32 x 32 fp32) are stored column-quad-major: element
// (i, j) at ((j / 4) * 32 + i) * 4 + j % 4, so that lanes that own rows move 512
// contiguous bytes per warp instruction.
// tile T (TRANS: its transpose) -> an operator; synchronise the warp before
template <bool TRANS>
static __device__ __noinline__ void store_op_tile(float* dst, const float* T, int lane) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float4 x;
    if (TRANS)
      x = make_float4(T[swz(4 * k, lane)], T[swz(4 * k + 1, lane)], T[swz(4 * k + 2, lane)], T[swz(4 * k + 3, lane)]);
    else
      x = reinterpret_cast<const float4*>(T + lane * 32)[k ^ (lane & 7)];
    d4[k * 32 + lane] = x;
  }
}
// an operator -> tile T by cp.async (part of the lane's next commit group)
__device__ __forceinline__ void cp_op_async(float* T, const float* src, int lane) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(T + lane * 32 + ((k ^ (lane & 7)) << 2)));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + (k * 32 + lane) * 4) : "memory");
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {   // at most N of this lane's groups still in flight
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// rows [0, nrows) x columns [0, ncols) of tile T, times scale -> row-major global
// matrix (coalesced when ncols == 32, as load_mat).  Synchronise the warp before.
static __device__ __noinline__ void store_mat(float* dst, const float* T, int nrows, int ncols, float scale,
                                          int lane) {
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int f = 32 * k + lane, row = f >> 3, q = f & 7;
      if (row < nrows) {
        const float4 x = reinterpret_cast<const float4*>(T + row * 32)[q ^ (row & 7)];
        reinterpret_cast<float4*>(dst)[f] = make_float4(x.x * scale, x.y * scale, x.z * scale, x.w * scale);
      }
    }
  } else {
    float v[32];
    ld_row(v, T, lane);
    if (lane < nrows) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) dst[(size_t)lane * ncols + j] = v[j] * scale;
    }
  }
}

struct ChunkId {
  long long q, bh;
  int b, h, c;
};
__device__ __forceinline__ ChunkId chunk_id(const Dims& d, long long q) {
  ChunkId id;
  id.q = q;
  id.c = (int)(q % d.C);
  id.bh = q / d.C;
  id.h = (int)(id.bh % d.H);
  id.b = (int)(id.bh / d.H);
  return id;
}

__device__ __forceinline__ float series_norm(const unsigned long long* cmax, const ChunkId& id, int C, int lane) {
  unsigned long long key = 0ull;
  for (int cc = lane; cc < C; cc += 32) {
    const unsigned long long x = cmax[id.bh * C + cc];
    key = x > key ? x : key;
  }
  key = warp_max_u64(key);
  return fmaxf(unpack_norm(key), kNormClamp);
}

__device__ __forceinline__ uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32_acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- warp-level tile GEMM on tensor cores (mma.sync m16n8k8 TF32) ----
//
// C[M x 32] (=|+=) alpha * op(A)[M x K] op(B)[K x 32], all swizzled tiles (rows of
// 32 floats; "tall" operands are consecutive tiles, i.e. more rows):
//   op(A)(i,k) = TA ? A[(i >> 5) * SA + swz(k, i & 31)]   (A stored K x M in 32-col blocks)
//                   : A[(k >> 5) * SA + swz(i, k & 31)]   (A stored M x K in 32-col blocks)
//   op(B)(k,j) = TB ? B[swz(j, k)]  (B stored 32 x K, K <= 32) : B[swz(k, j)]  (tall)
//   C(i,j)     = C[swz(i, j)]
// Operands are split x = hi + lo with hi = x with its low 13 mantissa bits cleared
// (exactly a tf32 value) and lo = x - hi (exact); the TF32 MMA reads the top 19 bits
// of lo.  a*b ~= hi_a hi_b + hi_a lo_b + lo_a hi_b has ~2^-20 relative error, i.e.
// fp32-level products, at two ALU ops per operand value.  SPLIT = false uses hi only.
// C may not alias A or B.  All 32 lanes must call.
__device__ __forceinline__ uint32_t tf32_rn(float x) {
  return (__float_as_uint(x) + 0x1000u) & 0xffffe000u;   // nearest, ties away from zero
}
__device__ __forceinline__ void split_trunc(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// Not inlined: one copy per shape keeps the kernels small enough for the
// instruction cache (inlining every call site made instruction fetch the main stall).
// SA_ / SB_: split that operand (an operand holding bf16 values is exact in tf32 and
// is passed unsplit).  RN_: round unsplit operands to the nearest tf32 value
// (bits + 0x1000, low 13 bits cleared; exact values stay exact) instead of
// letting the MMA truncate them.  Two 16-row blocks are processed together so that they share
// the B fragments; M is a multiple of 32.  kn (a multiple of 8, <= K): only the first
// kn of the K terms are summed (the rest are known zero: padding past r).
template <int M, int K, bool TA, bool TB, bool ACC, bool SA_, bool SB_, bool RN_ = false>
__device__ __noinline__ void wmm2(float* __restrict__ C, const float* __restrict__ A, int SA,
                                  const float* __restrict__ B, float alpha, int kn = K) {
  static_assert(M % 32 == 0 && K % 8 == 0, "tile shape");
  static_assert(!TB || K <= 32, "transposed B holds 32 x K");
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int g2 = g >> 2, g3 = g & 3;
#pragma unroll 1
  for (int i0 = 0; i0 < M; i0 += 32) {
    float d[2][4][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int n = 0; n < 4; ++n) d[h][n][0] = d[h][n][1] = d[h][n][2] = d[h][n][3] = 0.f;
    // not unrolled: each product shape is its own function and the chunk kernels
    // stall on instruction fetch, so the smallest copies run fastest (backward at
    // B=8, H=12, L=2048, P=64, r=32: full unroll 0.2105 ms, by 2 0.2035 ms, none
    // 0.2012 ms)
#pragma unroll 1
    for (int k0 = 0; k0 < kn; k0 += 8) {
      if ((k0 & 15) == 0) sched_fence();
      const int kc = (k0 & 31) >> 2;         // 16-byte chunk of column ka; kb is kc + 1
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ra = i0 + 16 * h + g, rb = ra + 8;
        float av[4];
        if (TA) {
          // A(i,k) = T[(i>>5)*SA + k*32 + ((((i&31)>>2) ^ (k&7)) << 2) + (i&3)], k&7 = t4 (+4)
          const int ca = (((ra & 31) >> 2) ^ t4) << 2, cb = (((rb & 31) >> 2) ^ t4) << 2;
          const int ca4 = (((ra & 31) >> 2) ^ (t4 + 4)) << 2, cb4 = (((rb & 31) >> 2) ^ (t4 + 4)) << 2;
          const float* Pa = A + (ra >> 5) * SA + g3;
          const float* Pb = A + (rb >> 5) * SA + g3;
          av[0] = Pa[(k0 + t4) * 32 + ca];
          av[1] = Pb[(k0 + t4) * 32 + cb];
          av[2] = Pa[(k0 + t4 + 4) * 32 + ca4];
          av[3] = Pb[(k0 + t4 + 4) * 32 + cb4];
        } else {
          const float* P0 = A + (k0 >> 5) * SA + t4;
          const int sa = (kc ^ g) << 2, sb = ((kc + 1) ^ g) << 2;
          av[0] = P0[ra * 32 + sa];
          av[1] = P0[rb * 32 + sa];
          av[2] = P0[ra * 32 + sb];
          av[3] = P0[rb * 32 + sb];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (SA_) {
            split_trunc(av[u], ah[h][u], al[h][u]);
          } else {
            ah[h][u] = RN_ ? tf32_rn(av[u]) : __float_as_uint(av[u]);
            al[h][u] = 0u;
          }
        }
      }
      uint32_t bh[4][2], bl[4][2];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        float b0, b1;
        if (TB) {
          const float* Q = B + (n * 8 + g) * 32 + t4;
          b0 = Q[(kc ^ g) << 2];
          b1 = Q[((kc + 1) ^ g) << 2];
        } else {
          const int cc = 2 * n + g2;
          b0 = B[(k0 + t4) * 32 + ((cc ^ t4) << 2) + g3];
          b1 = B[(k0 + t4 + 4) * 32 + ((cc ^ (t4 + 4)) << 2) + g3];
        }
        if (SB_) {
          split_trunc(b0, bh[n][0], bl[n][0]);
          split_trunc(b1, bh[n][1], bl[n][1]);
        } else {
          bh[n][0] = RN_ ? tf32_rn(b0) : __float_as_uint(b0);
          bh[n][1] = RN_ ? tf32_rn(b1) : __float_as_uint(b1);
          bl[n][0] = bl[n][1] = 0u;
        }
      }
      // term-major issue order: consecutive MMAs update different accumulators, so
      // the three terms of one accumulator never wait on each other back to back
      if (SA_) {
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int h = 0; h < 2; ++h) mma_tf32_acc(d[h][n], al[h], bh[n][0], bh[n][1]);
      }
      if (SB_) {
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int h = 0; h < 2; ++h) mma_tf32_acc(d[h][n], ah[h], bl[n][0], bl[n][1]);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h) mma_tf32_acc(d[h][n], ah[h], bh[n][0], bh[n][1]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ra = i0 + 16 * h + g, rb = ra + 8;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        // C(r, col) for col = n*8 + 2*t4 (+1): chunk (2n + (t4 >> 1)) ^ g, word (2*t4) & 3 (+1)
        const int cw = ((((2 * n + (t4 >> 1)) ^ g) << 2) | ((2 * t4) & 3));
        float* c0 = C + ra * 32 + cw;
        float* c1 = C + rb * 32 + cw;
        if (ACC) {
          c0[0] += alpha * d[h][n][0];
          c0[1] += alpha * d[h][n][1];
          c1[0] += alpha * d[h][n][2];
          c1[1] += alpha * d[h][n][3];
        } else {
          c0[0] = alpha * d[h][n][0];
          c0[1] = alpha * d[h][n][1];
          c1[0] = alpha * d[h][n][2];
          c1[1] = alpha * d[h][n][3];
        }
      }
    }
  }
}

// wmm2 with bf16 operand halves on the m16n8k16 MMA: x = hi + lo with hi = bf16(x)
// and lo = bf16(x - hi) (~2^-16 relative, the precision of the tcgen05 chunk
// products), a*b ~= hi_a hi_b + hi_a lo_b + lo_a hi_b.  Half the MMAs of the TF32
// split for the same K (16 per instruction instead of 8); for the bf16-only chunk
// kernels.  Same operand forms, tile layout and alpha / ACC semantics as wmm2; kn
// is rounded up to a multiple of 16 (the extra terms are the zero padding).
__device__ __forceinline__ void mma_bf16_acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x0, x1) -> bf16 pairs hi (x0 in the low half) and lo = the remainders
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int M, int K, bool TA, bool TB, bool ACC>
__device__ __noinline__ void wmm2b(float* __restrict__ C, const float* __restrict__ A, int SA,
                                   const float* __restrict__ B, float alpha, int kn = K) {
  static_assert(M % 32 == 0 && K % 16 == 0, "tile shape");
  static_assert(!TB || K <= 32, "transposed B holds 32 x K");
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int kr = (kn + 15) & ~15;
  // op(A)(i, k) and op(B)(k, j) as in wmm2
  const auto opA = [&](int i, int k) -> float {
    return TA ? A[(i >> 5) * SA + swz(k, i & 31)] : A[(k >> 5) * SA + swz(i, k & 31)];
  };
  const auto opB = [&](int k, int j) -> float { return TB ? B[swz(j, k)] : B[swz(k, j)]; };
#pragma unroll 1
  for (int i0 = 0; i0 < M; i0 += 32) {
    float d[2][4][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int n = 0; n < 4; ++n) d[h][n][0] = d[h][n][1] = d[h][n][2] = d[h][n][3] = 0.f;
#pragma unroll 1
    for (int k0 = 0; k0 < kr; k0 += 16) {
      sched_fence();
      const int c0 = k0 + 2 * t4;
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ra = i0 + 16 * h + g, rb = ra + 8;
        split_bf16x2(opA(ra, c0), opA(ra, c0 + 1), ah[h][0], al[h][0]);
        split_bf16x2(opA(rb, c0), opA(rb, c0 + 1), ah[h][1], al[h][1]);
        split_bf16x2(opA(ra, c0 + 8), opA(ra, c0 + 9), ah[h][2], al[h][2]);
        split_bf16x2(opA(rb, c0 + 8), opA(rb, c0 + 9), ah[h][3], al[h][3]);
      }
      uint32_t bh[4][2], bl[4][2];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int j = n * 8 + g;
        split_bf16x2(opB(c0, j), opB(c0 + 1, j), bh[n][0], bl[n][0]);
        split_bf16x2(opB(c0 + 8, j), opB(c0 + 9, j), bh[n][1], bl[n][1]);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h) mma_bf16_acc(d[h][n], al[h], bh[n][0], bh[n][1]);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h) mma_bf16_acc(d[h][n], ah[h], bl[n][0], bl[n][1]);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h) mma_bf16_acc(d[h][n], ah[h], bh[n][0], bh[n][1]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ra = i0 + 16 * h + g, rb = ra + 8;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int cw = ((((2 * n + (t4 >> 1)) ^ g) << 2) | ((2 * t4) & 3));
        float* c0p = C + ra * 32 + cw;
        float* c1p = C + rb * 32 + cw;
        if (ACC) {
          c0p[0] += alpha * d[h][n][0];
          c0p[1] += alpha * d[h][n][1];
          c1p[0] += alpha * d[h][n][2];
          c1p[1] += alpha * d[h][n][3];
        } else {
          c0p[0] = alpha * d[h][n][0];
          c0p[1] = alpha * d[h][n][1];
          c1p[0] = alpha * d[h][n][2];
          c1p[1] = alpha * d[h][n][3];
        }
      }
    }
  }
}

// Product of two fp32 tiles:
//   FAST = false: 3-term split, fp32-level products (what the kernels use);
//   FAST = true:  one TF32 product of round-to-nearest operands, ~2^-11 relative
//     per product.  Through the chunk algebra that is ~1.5e-3 at B=8, H=12,
//     L=2048, r=32 numerics, but with power_K = 3 and 32-token chunks the backward reached the
//     2e-2 bf16 bar, so it is not used.
template <bool FAST, int M, int K, bool TA, bool TB, bool ACC>
__device__ __forceinline__ void wmmp(float* C, const float* A, int SA, const float* B, float alpha, int kn = K) {
  if constexpr (FAST) {
    wmm2<M, K, TA, TB, ACC, false, false, true>(C, A, SA, B, alpha, kn);
  } else {
    wmm2<M, K, TA, TB, ACC, true, true>(C, A, SA, B, alpha, kn);
  }
}

}  // namespace wpc
}  // namespace ska
