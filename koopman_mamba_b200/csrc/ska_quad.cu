// ska_quad.cu -- chunk-operator forward for ranks 32 < r <= 64: one CTA of four
// warps per (batch, head, chunk).
//
// A 64 x 64 matrix is four of the warp kernels' swizzled 32 x 32 fp32 tiles,
// stored column-block major: block (bi, bj) (rows 32 bi.., columns 32 bj..) at
// tile 2 bj + bi.  Then a column block is two consecutive tiles, which the warp
// tile products (wmmp) read as one "tall" operand of 64 rows, and the two tiles of
// a row block are 2 tiles apart.  A P x 64 matrix (P <= 64) is NPB row blocks by
// two column blocks, block (pb, bj) at tile bj * NPB + pb.  Rows and columns past
// r hold the usual padding (identity on the Gram factor, zero elsewhere).
//
// Per chunk (same algebra as the warp kernels, KLF/koopman_lm/ska.py:136-186):
//   Gn = sym(G) / m^2 + ridge I        blocked Cholesky, by warp 0:
//     L11 = chol(Gn11), Li11 = L11^{-1}             (chol_inv32)
//     L21 = Gn21 Li11^T,  Gn22' = Gn22 - L21 L21^T
//     L22 = chol(Gn22'), Li22 = L22^{-1}            (chol_inv32)
//     Li21 = -Li22 L21 Li11
//   (a non-positive pivot in either block refactors the whole Gram matrix with
//    1e-4 added to its diagonal, ska.py:140-145: the blocked pivots are those of
//    the unblocked factorisation)
//   S = Li^T Li, A0 = Mn S                       one output block per warp
//   sigma: 6 power iterations (ska.py:41-58)     warps 0 and 1, a row per lane
//   A = clamp(gamma, 1, 1.5) / max(sigma, 1) A0,  A^K,  U = A^K Li,  V = Li^T U
//   W / m = C V / m^2                            one output block per warp
// and writes W / m as the bf16 hi / lo planes that k_readout_tc multiplies into
// the tokens (the readout is not done here).  Given a kept-operator array, it
// also copies Li, S, A0, A0^K, U and V out for the backward (k_bwd_chunk_q, below).
#include "ska_warp.cuh"

namespace ska {
namespace quad {

using namespace wpc;

constexpr int kThreads4 = 128;
constexpr int kTile = 1024;
constexpr int kRegion = 4 * kTile;   // one 64 x 64 matrix

__device__ __forceinline__ float* blk(float* M, int bi, int bj) { return M + ((bj << 1) | bi) * kTile; }

// tile T <- rows [0, nrows) x columns [0, ncols) of a global matrix with row stride
// ld (floats), zero elsewhere; by cp.async (the lane's next commit group) when the
// source rows are 16-byte aligned pieces, else by plain loads (then synchronise
// the warp before reading)
__device__ __forceinline__ void fetch_block(float* T, const float* src, int ld, int nrows, int ncols, int lane) {
  const bool vec = (ld & 3) == 0 && (ncols & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  if (vec) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int f = 32 * k + lane, row = f >> 3, q = f & 7;
      const bool ok = row < nrows && 4 * q < ncols;
      const float* s = src + (ok ? (size_t)row * ld + 4 * q : 0);
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(T + row * 32 + ((q ^ (row & 7)) << 2)));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(s), "r"(ok ? 16 : 0) : "memory");
    }
  } else {
    float v[32];
    const bool rv = lane < nrows;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (rv && j < ncols) ? __ldg(src + (size_t)lane * ld + j) : 0.f;
    st_row(T, lane, v);
  }
}

// the 64 x 64 record block starting at `src` (row stride r) -> region M
__device__ __forceinline__ void fetch_square(float* M, const float* src, int r, int lane) {
#pragma unroll
  for (int bj = 0; bj < 2; ++bj)
#pragma unroll
    for (int bi = 0; bi < 2; ++bi)
      fetch_block(blk(M, bi, bj), src + (size_t)(32 * bi) * r + 32 * bj, r, r - 32 * bi, r - 32 * bj, lane);
}

// G (r x r, row stride r, raw) read straight from the chunk record, as 32 x 32
// blocks: row(v, bi, bj) = row `lane` of block (bi, bj), col(v, bi, bj) = its
// column `lane`; zero past r.  (rec is 16-byte aligned and r % 8 == 0.)
struct GlobalGram {
  const float* G;
  int r;
  __device__ __forceinline__ void row(float (&v)[32], int bi, int bj, int lane) const {
    const int i = 32 * bi + lane, c0 = 32 * bj;
    const bool rv = i < r;
    const float4* p4 = reinterpret_cast<const float4*>(G + (size_t)(rv ? i : 0) * r + c0);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const bool ok = rv && c0 + 4 * k < r;
      const float4 x = ok ? __ldg(p4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * k] = x.x;
      v[4 * k + 1] = x.y;
      v[4 * k + 2] = x.z;
      v[4 * k + 3] = x.w;
    }
  }
  __device__ __forceinline__ void col(float (&v)[32], int bi, int bj, int lane) const {
    const int j = 32 * bj + lane, r0 = 32 * bi;
    const bool cv = j < r;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (cv && r0 + i < r) ? __ldg(G + (size_t)(r0 + i) * r + j) : 0.f;
  }
};

// The blocked Cholesky + inverse of one chunk's Gram matrix by one warp:
//   L11 = chol(Gn11), Li11 = L11^{-1}             (chol_inv32_bc)
//   L21 = Gn21 Li11^T,  Gn22' = Gn22 - L21 L21^T
//   L22 = chol(Gn22'), Li22 = L22^{-1}            (chol_inv32_bc, r - 32 steps)
//   Li21 = -Li22 L21 Li11
// with Gn = sym(G) / m^2 + (ridge + jit) I and identity padding past r.  Returns
// false (uniformly) when a pivot is not positive (the blocked pivots are those of
// the unblocked factorisation).  Li11, Li21, Li22: output tiles (Li12 is zero);
// T0, T1, T2: scratch tiles; cb: 32 floats (16-byte aligned) for the broadcasts.
__device__ bool blocked_factor(const Dims& d, const GlobalGram& G, float* Li11, float* Li21, float* Li22, float* T0,
                               float* T1, float* T2, float im2, float jit, float* cb, int lane) {
  const int r = d.r;
  float g[32], x[32], a[32], b[32];
  // block 11
  G.row(a, 0, 0, lane);
  G.col(b, 0, 0, lane);
  build_gram_row(g, a, b, lane, 32, im2, d.ridge, jit);
  if (!chol_inv32_bc(g, x, cb, lane)) return false;
  st_col<32>(Li11, lane, x);                                      // Li11 rows
  // Gn21 (row 32 + lane, column j): (G21 + G12^T) / 2 / m^2
  G.row(a, 1, 0, lane);
  G.col(b, 0, 1, lane);
  const bool row_ok = 32 + lane < r;
#pragma unroll
  for (int j = 0; j < 32; ++j) a[j] = row_ok ? 0.5f * (a[j] * im2 + b[j] * im2) : 0.f;
  st_row(T0, lane, a);
  // Gn22 (with identity padding past r)
  G.row(a, 1, 1, lane);
  G.col(b, 1, 1, lane);
  build_gram_row(g, a, b, lane, r - 32, im2, d.ridge, jit);
  st_row(T2, lane, g);
  __syncwarp();
  wmmp<false, 32, 32, false, true, false>(T1, T0, kTile, Li11, 1.f);     // L21 = Gn21 Li11^T
  __syncwarp();
  wmmp<false, 32, 32, false, true, true>(T2, T1, kTile, T1, -1.f);       // Gn22 - L21 L21^T
  __syncwarp();
  ld_row(g, T2, lane);
  if (!chol_inv32_bc<true>(g, x, cb, lane, r - 32)) return false;
  st_col<32>(Li22, lane, x);                                      // Li22 rows
  __syncwarp();
  wmmp<false, 32, 32, false, false, false>(T0, T1, kTile, Li11, 1.f);    // L21 Li11 (Gn21 is dead)
  __syncwarp();
  wmmp<false, 32, 32, false, false, false>(Li21, Li22, kTile, T0, -1.f); // Li21
  __syncwarp();
  return true;
}

// ---------------------------------------------------------------------------
// k_factor_q: the blocked Cholesky + inverse of every chunk, one warp per chunk,
// eight warps per SM (six 4 KB tiles of shared memory each), ahead of the
// four-warp operator kernel: there the factorisation ran on one warp while the
// other three waited at the next block barrier (~38K of the ~92K cycles of a
// chunk at r = 64).  Writes Li's three non-zero 32 x 32 tiles (Li11, Li21, Li22,
// as the operator kernel holds them in shared memory) and the jitter flags
// (ska.py:140-145: a non-positive pivot refactors with 1e-4 added to the
// diagonal; bit 1 when that fails too).
// ---------------------------------------------------------------------------
constexpr int kFacWarps = 4;
constexpr int kFacFloats = 6 * kTile + 32;   // per warp: Li11, Li21, Li22, T0..T2, the broadcast row

__global__ void __launch_bounds__(kFacWarps * 32, 2) k_factor_q(Dims d, const float* __restrict__ stats,
                                                                const unsigned long long* __restrict__ cmax,
                                                                float* __restrict__ lis, int* __restrict__ flags_out) {
  extern __shared__ float4 sm4[];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long q = (long long)blockIdx.x * kFacWarps + w;
  if (q >= (long long)d.B * d.H * d.C) return;   // warp-uniform; no block barriers below
  float* base = reinterpret_cast<float*>(sm4) + (size_t)w * kFacFloats;
  float* L11 = base;
  float* L21 = base + kTile;
  float* L22 = base + 2 * kTile;
  float* T0 = base + 3 * kTile;
  float* T1 = base + 4 * kTile;
  float* T2 = base + 5 * kTile;
  float* cb = base + 6 * kTile;
  const ChunkId id = chunk_id(d, q);
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const GlobalGram G{stats + q * d.SW, d.r};
  int flag = 0;
  if (!blocked_factor(d, G, L11, L21, L22, T0, T1, T2, im2, 0.f, cb, lane)) {
    flag = 1;
    if (!blocked_factor(d, G, L11, L21, L22, T0, T1, T2, im2, kJitter, cb, lane)) flag |= 2;
  }
  if (lane == 0) flags_out[q] = flag;
  __syncwarp();
  float* dst = lis + q * (long long)(3 * kTile);
  const float4* src4[3] = {reinterpret_cast<const float4*>(L11), reinterpret_cast<const float4*>(L21),
                           reinterpret_cast<const float4*>(L22)};
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float4* g4 = reinterpret_cast<float4*>(dst + t * kTile);
#pragma unroll
    for (int k = 0; k < 8; ++k) g4[32 * k + lane] = src4[t][32 * k + lane];
  }
}

// tile t of a 64 x 64 region -> the same tile of a kept operator in global memory
// (verbatim: the backward copies it back as it is), 16 bytes per lane and step
// The backward operator kernel's products: bf16 hi / lo operand halves on the
// m16n8k16 MMA (wmm2b, ~2^-16 relative, as the tcgen05 chunk products; half the
// MMAs of the TF32 split: k_bwd_chunk_q 0.925 -> 0.874 ms at the r = 48 layer).
// The forward keeps the TF32 split (wmmp): there the MMAs are not what limits it
// (no change with wmm2b).
template <int M, int K, bool TA, bool TB, bool ACC>
__device__ __forceinline__ void qmm(float* C, const float* A, int SA, const float* B, float alpha, int kn = K) {
  wmm2b<M, K, TA, TB, ACC>(C, A, SA, B, alpha, kn);
}

__device__ __forceinline__ void keep_tile(float* dst, const float* M, int t, int lane) {
  const float4* s = reinterpret_cast<const float4*>(M + t * kTile);
  float4* g = reinterpret_cast<float4*>(dst + t * kTile);
#pragma unroll
  for (int k = 0; k < 8; ++k) g[32 * k + lane] = s[32 * k + lane];
}

// A0 = Mn S etc.: out block (bi, bj) = alpha X(bi, :) Y(:, bj) for 64 x 64 X, Y
// (kn: the first kn of the 64 K terms; past r they are zero)
__device__ __forceinline__ void mul_block(float* out, float* X, float* Y, int bi, int bj, float alpha, int kn) {
  wmmp<false, 32, 64, false, false, false>(blk(out, bi, bj), blk(X, bi, 0), 2 * kTile, Y + bj * 2 * kTile, alpha,
                                           kn);
}

// sigma_max estimate of ska.py:41-58 for the 64 x 64 matrix A (region), by warps
// 0 and 1 (lane: row 32 w + lane, held in registers); the same arithmetic as
// power_sigma32: 6 iterations from v = 1/sqrt(r), x / max(||x||, 1e-8) taken as
// x * min(rsqrt(||x||^2), 1e8).  vsh: 64 floats; part: 2 x 64 floats; red: 2 floats.
// Named barrier 1 (64 threads).
__device__ __forceinline__ void bar64() { asm volatile("bar.sync 1, 64;" ::: "memory"); }

__device__ float power_sigma64(float* A, float* vsh, float* part, float* red, int r, int w, int lane) {
  float a0[32], a1[32];
  ld_row(a0, blk(A, w, 0), lane);
  ld_row(a1, blk(A, w, 1), lane);
  if (w == 0) {
    const float v0 = rsqrtf((float)r);
    vsh[lane] = lane < r ? v0 : 0.f;
    vsh[32 + lane] = 32 + lane < r ? v0 : 0.f;
  }
  bar64();
  float u = 0.f;
#pragma unroll 1
  for (int it = 0; it <= kPowerIters; ++it) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      s0 = fmaf(a0[j], vsh[j], s0);
      s1 = fmaf(a0[j + 1], vsh[j + 1], s1);
      s2 = fmaf(a1[j], vsh[32 + j], s2);
      s3 = fmaf(a1[j + 1], vsh[33 + j], s3);
    }
    u = (s0 + s1) + (s2 + s3);
    const float uu = warp_sum32(u * u);
    if (lane == 0) red[w] = uu;
    bar64();
    const float nu = red[0] + red[1];
    if (it == kPowerIters) return sqrtf(nu);
    u *= fminf(rsqrtf(nu), 1.f / kPowerEps);
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) t[i] = u * a0[i];
    const float p0 = reduce_scatter32(t, lane);
#pragma unroll
    for (int i = 0; i < 32; ++i) t[i] = u * a1[i];
    const float p1 = reduce_scatter32(t, lane);
    part[w * 64 + lane] = p0;
    part[w * 64 + 32 + lane] = p1;
    bar64();
    const float w0 = part[lane] + part[64 + lane], w1 = part[32 + lane] + part[96 + lane];
    const float nw = warp_sum32(w0 * w0 + w1 * w1);
    const float sc = fminf(rsqrtf(nw), 1.f / kPowerEps);
    bar64();                                   // every lane has read red and part
    if (w == 0) {
      vsh[lane] = w0 * sc;
      vsh[32 + lane] = w1 * sc;
    }
    bar64();
  }
  return 0.f;   // not reached
}

template <int NPB>
__global__ void __launch_bounds__(kThreads4, 3) k_fwd_chunk_q(Dims d, const float* __restrict__ gamma_p,
                                                              const float* __restrict__ stats,
                                                              const unsigned long long* __restrict__ cmax,
                                                              float* __restrict__ invs_out,
                                                              const float* __restrict__ lis,
                                                              float* __restrict__ ops_out,
                                                              unsigned char* __restrict__ wm_out) {
  extern __shared__ float4 sm4[];
  float* R0 = reinterpret_cast<float*>(sm4);   // S, then A^K / U / V / spare
  float* RLi = R0 + kRegion;                   // Li, then W / m
  float* RA = RLi + kRegion;                   // A0 / A
  float* RK = RA + kRegion;                    // Mn, then A^K
  __shared__ float vsh[64], part[128], red[2];
  __shared__ float s_sigma;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;
  const ChunkId id = chunk_id(d, q);
  const int r = d.r, P = d.P;
  const float* rec = stats + q * d.SW;
  // kept operators (when the caller keeps them): each warp writes tile w of each
  float* opq = ops_out ? ops_out + q * (long long)(kNumOps * kQOpFloats) : nullptr;

  // Li (k_factor_q): warps 0-2 copy its three non-zero tiles in, warp 3 zeroes
  // block (0, 1); M from the record (warp 1)
  {
    const float* src = lis + q * (long long)(3 * kTile);
    if (w < 3) {
      float* dst = RLi + (w == 2 ? 3 : w) * kTile;           // tiles (0, 0), (1, 0), (1, 1)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t da = static_cast<uint32_t>(__cvta_generic_to_shared(dst + (32 * k + lane) * 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(da), "l"(src + w * kTile + (32 * k + lane) * 4)
                     : "memory");
      }
    } else {
      float z[32];
      zero(z);
      st_row(blk(RLi, 0, 1), lane, z);
    }
  }
  if (w == 1) fetch_square(RK, rec + r * r, r, lane);      // M
  cp_async_commit();
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  cp_async_wait<0>();                                      // Li (and M on warp 1)
  __syncthreads();
  if (opq) keep_tile(opq + kQOpLi * kQOpFloats, RLi, w, lane);

  // ---- S = Li^T Li (block (0, 1) of Li is zero) ----
  {
    const int bi = w & 1, bj = w >> 1;
    float* out = blk(R0, bi, bj);
    if (bi == 0 && bj == 0)
      wmmp<false, 32, 64, true, false, false>(out, RLi, kTile, RLi, 1.f, r);
    else if (bi == 1 && bj == 0)
      wmmp<false, 32, 32, true, false, false>(out, blk(RLi, 1, 1), kTile, blk(RLi, 1, 0), 1.f, r - 32);
    else if (bi == 0)
      wmmp<false, 32, 32, true, false, false>(out, blk(RLi, 1, 0), kTile, blk(RLi, 1, 1), 1.f, r - 32);
    else
      wmmp<false, 32, 32, true, false, false>(out, blk(RLi, 1, 1), kTile, blk(RLi, 1, 1), 1.f, r - 32);
  }
  __syncthreads();
  if (opq) keep_tile(opq + kQOpS * kQOpFloats, R0, w, lane);
  // ---- A0 = Mn S ----
  mul_block(RA, RK, R0, w & 1, w >> 1, im2, r);
  __syncthreads();
  if (opq) keep_tile(opq + kQOpA0 * kQOpFloats, RA, w, lane);
  // ---- spectral norm (warps 0, 1) while warps 2, 3 form A0^K ----
  // A = kk A0 with kk = clamp(gamma, 1, 1.5) / max(sigma, 1), so A^K = kk^K A0^K:
  // the power of the unscaled A0 does not wait for sigma, and kk^K goes into the
  // alpha of the next product.  A0^K ping-pongs between RK (Mn, dead) and R0 (S, dead);
  // K = 0 gives the identity, K = 1 A0 itself.
  float* AK = RA;
  if (w < 2) {
    const float sg = power_sigma64(RA, vsh, part, red, r, w, lane);
    if (tid == 0) {
      s_sigma = sg;
      invs_out[q] = 1.f / fmaxf(sg, 1.f);   // (k_factor_q wrote the flags)
    }
  } else if (d.K == 0) {
    float t[32];
#pragma unroll 1
    for (int bi = 0; bi < 2; ++bi) {
      const int bj = w - 2;
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = (bi == bj && j == lane) ? 1.f : 0.f;
      st_row(blk(RK, bi, bj), lane, t);
    }
  } else {
    const float* prev = RA;
    for (int s = 1; s < d.K; ++s) {
      float* out = (prev == RK) ? R0 : RK;
      const int bj = w - 2;   // warps 2, 3: column block 0, 1 (both row blocks)
      mul_block(out, const_cast<float*>(prev), RA, 0, bj, 1.f, r);
      mul_block(out, const_cast<float*>(prev), RA, 1, bj, 1.f, r);
      asm volatile("bar.sync 2, 64;" ::: "memory");   // warps 2, 3: the power is complete
      prev = out;
    }
  }
  if (d.K == 0) AK = RK;
  else {
    for (int s = 1; s < d.K; ++s) AK = (AK == RK) ? R0 : RK;
  }
  __syncthreads();
  if (opq) keep_tile(opq + kQOpA0K * kQOpFloats, AK, w, lane);
  const float kk = gs * (1.f / fmaxf(s_sigma, 1.f));     // as the backward forms it from invs
  float kkK = 1.f;
  for (int s = 0; s < d.K; ++s) kkK *= kk;
  // regions now: RLi = Li, AK in one of {RA, RK, R0}; A (RA) dead unless AK is RA
  float* cand[3] = {R0, RK, RA};
  float* RU = nullptr;
  float* RC = nullptr;
  for (int i = 0; i < 3; ++i) {
    if (cand[i] == AK) continue;
    if (!RU) RU = cand[i];
    else if (!RC) RC = cand[i];
  }
  // C rows (P x r, row stride r) into RC, overlapping the U product
  if (w == 2) {
#pragma unroll
    for (int bj = 0; bj < 2; ++bj)
#pragma unroll
      for (int pb = 0; pb < NPB; ++pb)
        fetch_block(RC + (bj * NPB + pb) * kTile, rec + 2 * r * r + (size_t)(32 * pb) * r + 32 * bj, r, P - 32 * pb,
                    r - 32 * bj, lane);
    cp_async_commit();
  }
  // ---- U = A^K Li = kk^K A0^K Li (Li block (0, 1) is zero) ----
  {
    const int bi = w & 1, bj = w >> 1;
    if (bj == 0)
      wmmp<false, 32, 64, false, false, false>(blk(RU, bi, 0), blk(AK, bi, 0), 2 * kTile, RLi, kkK, r);
    else
      wmmp<false, 32, 32, false, false, false>(blk(RU, bi, 1), blk(AK, bi, 1), kTile, blk(RLi, 1, 1), kkK, r - 32);
  }
  __syncthreads();
  if (opq) keep_tile(opq + kQOpU * kQOpFloats, RU, w, lane);
  // ---- V = Li^T U (into the A^K region, dead now) ----
  float* RV = AK;
  {
    const int bi = w & 1, bj = w >> 1;
    if (bi == 0)
      wmmp<false, 32, 64, true, false, false>(blk(RV, 0, bj), RLi, kTile, RU + bj * 2 * kTile, 1.f, r);
    else
      wmmp<false, 32, 32, true, false, false>(blk(RV, 1, bj), blk(RLi, 1, 1), kTile, blk(RU, 1, bj), 1.f, r - 32);
  }
  if (w == 2) cp_async_wait<0>();                          // C
  __syncthreads();
  if (opq) keep_tile(opq + kQOpV * kQOpFloats, RV, w, lane);
  // ---- W / m = C V / m^2 (into the Li region, dead now), then its bf16 planes ----
  float* RW = RLi;
  for (int t = w; t < 2 * NPB; t += 4) {
    const int pb = t % NPB, bj = t / NPB;
    float* out = RW + (bj * NPB + pb) * kTile;
    wmmp<false, 32, 64, false, false, false>(out, RC + pb * kTile, NPB * kTile, RV + bj * 2 * kTile, im2, r);
    __syncwarp();
    float u[32];
    ld_row(u, out, lane);
    const int p = 32 * pb + lane;
    if (p < P && wm_out) {
      unsigned char* wq = wm_out + (size_t)q * P * r * 4;
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        const int ng = 4 * bj + g4;
        if (8 * ng >= r) break;
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = u[8 * g4 + e];
        uint4 hi, lo;
        split_bf16x8(x, hi, lo);
        *reinterpret_cast<uint4*>(wq + (size_t)ng * P * 16 + (size_t)p * 16) = hi;
        *reinterpret_cast<uint4*>(wq + (size_t)P * r * 2 + (size_t)ng * P * 16 + (size_t)p * 16) = lo;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// backward for 32 < r <= 64 without the token pass (bf16 token tensors on the
// tensor-core path), from the operators the forward kept: one CTA of four warps
// per chunk, warp w owning output block (w & 1, w >> 1) = tile w of every product.
//
// dW' = sum_t dy_t zq_t^T comes from k_dw_tc and dzq from k_tok_bwd_tc (W / m
// planes), as for r <= 32.  The chain rule through W / m = C V / m^2, V = Li^T U,
// U = A^K Li, A = kk A0, A0 = Mn S, S = Li^T Li (KLF/koopman_lm/ska.py:136-186
// differentiated; the same steps as the warp kernel k_bwd_chunk_s):
//   dV = C^T dW' / m^2, m dCn = dW' V^T
//   dU = Li dV,          dLi  = U dV^T
//   dA^K = dU Li^T,      dLi += (A^K)^T dU
//   dA = dA^K A^T + A^T dA^K (K = 2), dA^K (K = 1), 0 (K = 0)
//   dMn = kk dA S,  dS = kk Mn^T dA,  dLi += Li (dS + dS^T)
//   Pm = tril(-tril(dLi) Li^T),  P' = (Pm + tril(Pm, -1)^T) / 2
//   dGn = sym(Li^T P' Li)
// with the d(max norm) share -(2 <dGn, Gn> + 2 <dMn, Mn> + <dCn, Cn> + <dQn, Qn>) / m
// and the d(gamma) share <dA, A> / gamma' (zero outside the clamp).  Seven 64 x 64
// regions (112 KB, two CTAs per SM); the kept operators arrive by cp.async into
// regions as they free up.
// ---------------------------------------------------------------------------
constexpr int kBwdRegions = 7;

// tile t of a kept operator -> tile t of region M (this lane's next commit group)
__device__ __forceinline__ void fetch_kept_tile(float* M, const float* src, int t, int lane) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(M + t * kTile + (32 * k + lane) * 4));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + t * kTile + (32 * k + lane) * 4)
                 : "memory");
  }
}

// rows [0, nrows) x columns [0, ncols) of tile T, times scale -> global matrix with
// row stride ld (16-byte pieces when the layout allows).  Synchronise the warp before.
__device__ __forceinline__ void store_block(float* dst, int ld, const float* T, int nrows, int ncols, float scale,
                                            int lane) {
  if (nrows <= 0 || ncols <= 0) return;
  if ((ld & 3) == 0 && (ncols & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int f = 32 * k + lane, row = f >> 3, q = f & 7;
      if (row < nrows && 4 * q < ncols) {
        const float4 x = reinterpret_cast<const float4*>(T + row * 32)[q ^ (row & 7)];
        *reinterpret_cast<float4*>(dst + (size_t)row * ld + 4 * q) =
            make_float4(x.x * scale, x.y * scale, x.z * scale, x.w * scale);
      }
    }
  } else {
    float v[32];
    ld_row(v, T, lane);
    if (lane < nrows) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) dst[(size_t)lane * ld + j] = v[j] * scale;
    }
  }
}

// out block (bi, bj) of 64 x 64 products (alpha folded in; ACC accumulates).  kn:
// the first kn (a multiple of 8) of the 64 K terms; past r (or P) they are
// zero, and every matrix here is zero between its valid and padding parts, so the
// valid part of the product does not change
template <bool ACC>
__device__ __forceinline__ void mm_nn(float* out, const float* X, const float* Y, int bi, int bj, float alpha,
                                      int kn) {
  qmm<32, 64, false, false, ACC>(blk(out, bi, bj), blk(const_cast<float*>(X), bi, 0), 2 * kTile,
                                         Y + bj * 2 * kTile, alpha, kn);   // X Y
}
template <bool ACC>
__device__ __forceinline__ void mm_tn(float* out, const float* X, const float* Y, int bi, int bj, float alpha,
                                      int kn) {
  qmm<32, 64, true, false, ACC>(blk(out, bi, bj), X + bi * 2 * kTile, kTile, Y + bj * 2 * kTile,
                                        alpha, kn);                        // X^T Y
}
template <bool ACC>
__device__ __forceinline__ void mm_nt(float* out, const float* X, const float* Y, int bi, int bj, float alpha,
                                      int kn) {
  float* Xm = const_cast<float*>(X);
  float* Ym = const_cast<float*>(Y);
  qmm<32, 32, false, true, ACC>(blk(out, bi, bj), blk(Xm, bi, 0), kTile, blk(Ym, bj, 0), alpha,
                                        min(kn, 32));   // X Y^T
  if (kn > 32)
    qmm<32, 32, false, true, true>(blk(out, bi, bj), blk(Xm, bi, 1), kTile, blk(Ym, bj, 1), alpha, kn - 32);
}

// tril of block (bi, bj) of a 64 x 64 matrix, in place, by the warp that owns it
__device__ __forceinline__ void tril_block(float* M, int bi, int bj, int lane) {
  float t[32];
  float* T = blk(M, bi, bj);
  ld_row(t, T, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (bi < bj || (bi == bj && j > lane)) t[j] = 0.f;
  __syncwarp();
  st_row(T, lane, t);
}

__device__ __forceinline__ float dot_block(const float* X, const float* Y, int bi, int bj, int lane) {
  float a[32], b[32];
  ld_row(a, blk(const_cast<float*>(X), bi, bj), lane);
  ld_row(b, blk(const_cast<float*>(Y), bi, bj), lane);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) s = fmaf(a[j], b[j], s);
  return s;
}

__global__ void __launch_bounds__(kThreads4, 2) k_bwd_chunk_q(Dims d, const float* __restrict__ gamma_p,
                                                              const float* __restrict__ stats,
                                                              const unsigned long long* __restrict__ cmax,
                                                              const float* __restrict__ invs_in,
                                                              const float* __restrict__ ops,
                                                              const float* __restrict__ dwraw,
                                                              float* __restrict__ dstats,
                                                              float* __restrict__ dmpart,
                                                              float* __restrict__ dgpart) {
  extern __shared__ float4 sm4[];
  float* R[kBwdRegions];
#pragma unroll
  for (int i = 0; i < kBwdRegions; ++i) R[i] = reinterpret_cast<float*>(sm4) + i * kRegion;
  float* red = reinterpret_cast<float*>(sm4) + kBwdRegions * kRegion;   // 8 floats
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int bi = w & 1, bj = w >> 1;   // this warp's block; its tile index is w
  const long long q = blockIdx.x;
  const ChunkId id = chunk_id(d, q);
  const int r = d.r, P = d.P;
  const float* rec = stats + q * d.SW;
  const float* opq = ops + q * (long long)(kNumOps * kQOpFloats);
  const float* dwq = dwraw + q * (long long)P * r;
  float* drec = dstats + q * d.SW;
  const int rows_r = r - 32 * bi, cols_r = r - 32 * bj, rows_p = P - 32 * bi;
  const int kp = (P + 7) & ~7;                       // K of the products over the P value rows

  // C -> R0, dW' -> R1, V -> R2 (group 0); Li -> R3, U -> R4 (group 1)
  fetch_block(blk(R[0], bi, bj), rec + 2 * r * r + (size_t)(32 * bi) * r + 32 * bj, r, rows_p, cols_r, lane);
  fetch_block(blk(R[1], bi, bj), dwq + (size_t)(32 * bi) * r + 32 * bj, r, rows_p, cols_r, lane);
  fetch_kept_tile(R[2], opq + kQOpV * kQOpFloats, w, lane);
  cp_async_commit();
  fetch_kept_tile(R[3], opq + kQOpLi * kQOpFloats, w, lane);
  fetch_kept_tile(R[4], opq + kQOpU * kQOpFloats, w, lane);
  cp_async_commit();
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const float gam = *gamma_p;
  const float gs = fminf(fmaxf(gam, 1.f), 1.5f);
  const bool gpass = gam >= 1.f && gam <= 1.5f;       // clamp passes gradients inclusively
  const float kk = gs * invs_in[q];
  float kkK = 1.f;
  for (int s = 0; s < d.K; ++s) kkK *= kk;
  cp_async_wait<1>();
  __syncthreads();

  // ---- dV = C^T dW' / m^2 -> R5,  TY = dW' V^T = m dCn -> R6 ----
  mm_tn<false>(R[5], R[0], R[1], bi, bj, im2, kp);
  mm_nt<false>(R[6], R[1], R[2], bi, bj, 1.f, r);
  __syncwarp();
  store_block(drec + 2 * r * r + (size_t)(32 * bi) * r + 32 * bj, r, blk(R[6], bi, bj), min(rows_p, 32),
              min(cols_r, 32), im2, lane);
  const float dmc = dot_block(R[6], R[0], bi, bj, lane);   // <TY, C> = m^2 <dCn, Cn>
  const float dmq = dot_block(R[2], R[5], bi, bj, lane);   // <V, dV> = <W, dW> = <dQn, Qn>
  cp_async_wait<0>();
  __syncthreads();
  // free: R0, R1, R2, R6.  A0^K -> R0, A0 -> R1 (group 2)
  fetch_kept_tile(R[0], opq + kQOpA0K * kQOpFloats, w, lane);
  fetch_kept_tile(R[1], opq + kQOpA0 * kQOpFloats, w, lane);
  cp_async_commit();

  // ---- dU = Li dV -> R2,  dLi = U dV^T -> R6 ----
  mm_nn<false>(R[2], R[3], R[5], bi, bj, 1.f, r);
  mm_nt<false>(R[6], R[4], R[5], bi, bj, 1.f, r);
  cp_async_wait<0>();
  __syncthreads();
  // free: R4 (U), R5 (dV).  S -> R4 (group 3)
  fetch_kept_tile(R[4], opq + kQOpS * kQOpFloats, w, lane);
  cp_async_commit();

  // ---- dLi += (A^K)^T dU,  dA^K = dU Li^T -> R5  (A^K = kk^K A0^K) ----
  mm_tn<true>(R[6], R[0], R[2], bi, bj, kkK, r);
  mm_nt<false>(R[5], R[2], R[3], bi, bj, 1.f, r);
  cp_async_wait<0>();
  __syncthreads();
  // free: R0 (A0^K), R2 (dU).  M -> R0 (group 4)
  fetch_block(blk(R[0], bi, bj), rec + r * r + (size_t)(32 * bi) * r + 32 * bj, r, rows_r, cols_r, lane);
  cp_async_commit();

  // ---- dA (A = kk A0) ----
  float* RdA = R[2];
  if (d.K >= 2) {
    // K = 2: dA^K A^T + A^T dA^K
    mm_nt<false>(R[2], R[5], R[1], bi, bj, kk, r);
    mm_tn<true>(R[2], R[1], R[5], bi, bj, kk, r);
  } else if (d.K == 1) {
    RdA = R[5];
  } else {
    float t[32];
    zero(t);
    st_row(blk(R[2], bi, bj), lane, t);
  }
  __syncwarp();
  const float dg = kk * dot_block(RdA, R[1], bi, bj, lane);   // <dA, A>
  cp_async_wait<0>();
  __syncthreads();
  float* RdS = (RdA == R[5]) ? R[2] : R[5];
  float* RdMn = R[1];                                          // A0 is dead

  // ---- dMn = kk dA S -> R1,  dS = kk Mn^T dA -> RdS ----
  mm_nn<false>(RdMn, RdA, R[4], bi, bj, kk, r);
  mm_tn<false>(RdS, R[0], RdA, bi, bj, kk * im2, r);
  __syncwarp();
  store_block(drec + r * r + (size_t)(32 * bi) * r + 32 * bj, r, blk(RdMn, bi, bj), min(rows_r, 32), min(cols_r, 32),
              im2, lane);
  const float dmm = im2 * dot_block(RdMn, R[0], bi, bj, lane);   // <dMn, Mn>
  __syncthreads();
  // free: R0 (M), R1 (dMn), R4 (S), RdA.  G -> R4 (group 5)
  fetch_block(blk(R[4], bi, bj), rec + (size_t)(32 * bi) * r + 32 * bj, r, rows_r, cols_r, lane);
  cp_async_commit();

  // ---- dS + dS^T -> R0 ----
  {
    float t[32], u[32];
    ld_row(t, blk(RdS, bi, bj), lane);
    ld_col<32>(u, blk(RdS, bj, bi), lane);
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] += u[j];
    st_row(blk(R[0], bi, bj), lane, t);
  }
  __syncthreads();
  // ---- dLi += Li (dS + dS^T); only tril(dLi) reaches L ----
  mm_nn<true>(R[6], R[3], R[0], bi, bj, 1.f, r);
  __syncwarp();
  tril_block(R[6], bi, bj, lane);
  __syncthreads();
  // ---- Pm = tril(-dLi Li^T) -> R1 ----
  mm_nt<false>(R[1], R[6], R[3], bi, bj, -1.f, r);
  __syncwarp();
  tril_block(R[1], bi, bj, lane);
  __syncthreads();
  // ---- P' = (Pm + tril(Pm, -1)^T) / 2 -> RdS (dS is dead) ----
  {
    float t[32], u[32];
    ld_row(t, blk(R[1], bi, bj), lane);
    ld_col<32>(u, blk(R[1], bj, bi), lane);
    const int I = 32 * bi + lane;
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] = 0.5f * ((32 * bj + j <= I) ? t[j] : u[j]);
    st_row(blk(RdS, bi, bj), lane, t);
  }
  __syncthreads();
  // ---- T1 = P' Li -> R0,  dGn = Li^T T1 -> R1 ----
  mm_nn<false>(R[0], RdS, R[3], bi, bj, 1.f, r);
  cp_async_wait<0>();                                          // G
  __syncthreads();
  mm_tn<false>(R[1], R[3], R[0], bi, bj, 1.f, r);
  __syncthreads();
  // ---- sym(dGn) / m^2 -> dstats; <dGn, Gn> ----
  float dmg = 0.f;
  {
    float t[32], u[32], gr[32], gc[32];
    ld_row(t, blk(R[1], bi, bj), lane);
    ld_col<32>(u, blk(R[1], bj, bi), lane);
    ld_row(gr, blk(R[4], bi, bj), lane);
    ld_col<32>(gc, blk(R[4], bj, bi), lane);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float gsym = 0.5f * (t[j] + u[j]);
      dmg = fmaf(gsym, 0.5f * (gr[j] + gc[j]) * im2, dmg);
      t[j] = gsym;
    }
    st_row(blk(R[6], bi, bj), lane, t);                        // dLi is dead
    __syncwarp();
    store_block(drec + (size_t)(32 * bi) * r + 32 * bj, r, blk(R[6], bi, bj), min(rows_r, 32), min(cols_r, 32), im2,
                lane);
  }
  const float tot = warp_sum32(2.f * dmg + 2.f * dmm + dmc * im2 + dmq);
  const float dgs = warp_sum32(dg);
  if (lane == 0) {
    red[w] = tot;
    red[4 + w] = dgs;
  }
  __syncthreads();
  if (tid == 0) {
    dmpart[q] = -((red[0] + red[1]) + (red[2] + red[3])) / m;
    dgpart[q] = gpass ? ((red[4] + red[5]) + (red[6] + red[7])) / gs : 0.f;
  }
}

}  // namespace quad

// 32 < r <= 64, r % 8 == 0, P <= 64: the four-warp chunk operators (readout elsewhere)
bool quad_path_ok(const Dims& d) { return d.r > 32 && d.r <= 64 && (d.r & 7) == 0 && d.P <= 64; }

size_t smem_fwd_chunk_q(const Dims&) { return (size_t)4 * quad::kRegion * sizeof(float); }

// the four-warp backward from kept operators: power_K <= 2
bool quad_bwd_ok(const Dims& d) { return quad_path_ok(d) && d.K <= 2; }

cudaError_t launch_bwd_chunk_q(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               const float* invs, const float* ops, const float* dwraw, float* dstats, float* dmpart,
                               float* dgpart, cudaStream_t st) {
  const size_t smem = (size_t)quad::kBwdRegions * quad::kRegion * sizeof(float) + 8 * sizeof(float);
  const long long n = (long long)d.B * d.H * d.C;
  cudaError_t e = cudaFuncSetAttribute(quad::k_bwd_chunk_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  quad::k_bwd_chunk_q<<<(unsigned)n, quad::kThreads4, smem, st>>>(d, gamma, stats, cmax, invs, ops, dwraw, dstats,
                                                                  dmpart, dgpart);
  return cudaGetLastError();
}

// lis: room for Li's three tiles per chunk (the factor kernel's output)
cudaError_t launch_fwd_chunk_q(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               float* invs, int* flags, float* lis, float* ops, unsigned char* wm, cudaStream_t st) {
  const size_t smem = smem_fwd_chunk_q(d);
  const long long n = (long long)d.B * d.H * d.C;
  cudaError_t e;
  {
    const size_t fsmem = (size_t)quad::kFacWarps * quad::kFacFloats * sizeof(float);
    if ((e = cudaFuncSetAttribute(quad::k_factor_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem)) !=
        cudaSuccess)
      return e;
    const unsigned fgrid = (unsigned)((n + quad::kFacWarps - 1) / quad::kFacWarps);
    quad::k_factor_q<<<fgrid, quad::kFacWarps * 32, fsmem, st>>>(d, stats, cmax, lis, flags);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (d.P <= 32) {
    if ((e = cudaFuncSetAttribute(quad::k_fwd_chunk_q<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
      return e;
    quad::k_fwd_chunk_q<1><<<(unsigned)n, quad::kThreads4, smem, st>>>(d, gamma, stats, cmax, invs, lis, ops, wm);
  } else {
    if ((e = cudaFuncSetAttribute(quad::k_fwd_chunk_q<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
      return e;
    quad::k_fwd_chunk_q<2><<<(unsigned)n, quad::kThreads4, smem, st>>>(d, gamma, stats, cmax, invs, lis, ops, wm);
  }
  return cudaGetLastError();
}

}  // namespace ska
