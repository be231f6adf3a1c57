// ska_warp.cu -- warp-per-chunk SKA chunk-operator kernels for rank r <= 32.
//
// One warp owns one (batch, head, chunk).  The Cholesky factor, the triangular
// inverse and the power iteration keep one matrix row per lane in registers and
// run on shuffles; every matrix product is a warp-level tensor-core tile GEMM
// (wmmp: mma.sync TF32 with a 3-term split, fp32-level products) on the warp's
// swizzled shared-memory tiles.  There are no block barriers.
//
// Same algebra as the CTA path in ska_exact.cu, written with
//   U = A^K Li,  V = Li^T U,  W = Cn V           (W = Cn Li^T A^K Li)
// so that the backward is, besides the token contractions, r x r products only:
//   dV = Cn^T dW, dCn = dW V^T, dU = Li dV, dLi = U dV^T + A^K^T dU,
//   dA^K = dU Li^T, then dA, dMn, dS, dLi and dGn as in the CTA path.
#include "ska_warp.cuh"

namespace ska {
namespace wpc {

// tokens stored as bf16 are exact in tf32, so the tensor-core products need not split them
template <typename IO> constexpr bool kIoExact = false;
template <> constexpr bool kIoExact<__nv_bfloat16> = true;

constexpr int kMaxWarps = 8;   // chunks (warps) per CTA, fewer when the tiles do not fit
constexpr size_t kSmemBudget = 227 * 1024;
constexpr int kTile = 1024;    // floats per 32 x 32 tile

// forward tiles per warp: T0..T3, TC (P rows: Cn, then Y), TW (P rows: W / m)
__host__ __device__ inline int fwd_tiles(int P) { return 4 + 2 * p_blocks(P); }
// backward tiles per warp: Li, A, AK, V, X, Y, W[NPB], DY[NPB], DW[NPB]
__host__ __device__ inline int bwd_tiles(int P) { return 6 + 3 * p_blocks(P); }

// features [f0, f0 + n) of token t (n <= 32), times `scale`; zero when !valid
template <typename IO>
__device__ __forceinline__ void ld_tok_row(float (&v)[32], const In& x, int b, int t, int h, int f0, int n,
                                           bool valid, float scale) {
  const IO* p = static_cast<const IO*>(x.p) + (long long)b * x.sb + (long long)(valid ? t : 0) * x.st +
                (long long)h * x.sh + f0;
  constexpr int kVec = 16 / sizeof(IO);          // elements per 16-byte load
  if (n == 32 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    uint4 raw[32 / kVec];
#pragma unroll
    for (int q = 0; q < 32 / kVec; ++q) raw[q] = __ldg(reinterpret_cast<const uint4*>(p) + q);
#pragma unroll
    for (int q = 0; q < 32 / kVec; ++q) {
      const IO* e = reinterpret_cast<const IO*>(&raw[q]);   // registers: plain reads only
#pragma unroll
      for (int u = 0; u < kVec; ++u) v[q * kVec + u] = valid ? to_float(e[u]) * scale : 0.f;
    }
  } else {
    float xv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) xv[j] = load_elem<IO>(p + (j < n ? j : 0));
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (valid && j < n) ? xv[j] * scale : 0.f;
  }
}

__device__ __forceinline__ void pack_store(float* dst, const float (&v)[32], int q, float scale) {
  *reinterpret_cast<float4*>(dst) = make_float4(v[4 * q] * scale, v[4 * q + 1] * scale, v[4 * q + 2] * scale,
                                                v[4 * q + 3] * scale);
}
__device__ __forceinline__ void pack_store(__nv_bfloat16* dst, const float (&v)[32], int q, float scale) {
  __nv_bfloat162 p[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) p[u] = __floats2bfloat162_rn(v[8 * q + 2 * u] * scale, v[8 * q + 2 * u + 1] * scale);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(p);
}

// features [f0, f0 + n) of token t <- v * scale (n <= 32), when valid
template <typename IO>
__device__ __forceinline__ void st_tok_row(const Out& x, int b, int t, int h, int f0, int n, bool valid,
                                           const float (&v)[32], float scale) {
  if (!valid) return;
  IO* p = static_cast<IO*>(x.p) + (long long)b * x.sb + (long long)t * x.st + (long long)h * x.sh + f0;
  constexpr int kVec = 16 / sizeof(IO);
  if (n == 32 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 32 / kVec; ++q) pack_store(p + q * kVec, v, q, scale);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n) store_elem<IO>(p + j, v[j] * scale);
  }
}

// this lane's row of the identity -> tile T
__device__ __forceinline__ void st_identity(float* T, int lane) {
  float e[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) e[j] = (j == lane) ? 1.f : 0.f;
  st_row(T, lane, e);
}

// Gram factor and inverse.  Loads the raw G (scratch tile Tg), builds Gn, factors
// it (jitter retry as ska.py:140-145, or jitter forced), and writes Li rows into TLi.
// Returns the jitter flags.
__device__ __forceinline__ int factor_and_invert(const Dims& d, const float* rec, int lane, float im2,
                                                 bool force_jitter, float* Tg, float* TLi, bool preloaded = false) {
  const int r = d.r;
  if (!preloaded) load_mat(Tg, rec, r, r, 1.f, lane);   // else Tg already holds G
  __syncwarp();
  float g[32], x[32];
  int flag = 0;
  {
    float grow[32], gcol[32];
    ld_row(grow, Tg, lane);
    ld_col<32>(gcol, Tg, lane);
    // attempt 0: plain (or jittered when forced); attempt 1: jittered (ska.py:140-145)
    bool jit = force_jitter;
#pragma unroll 1
    for (int attempt = 0; attempt < 2; ++attempt) {
      build_gram_row(g, grow, gcol, lane, r, im2, d.ridge, jit ? kJitter : 0.f);
      if (jit) flag |= 1;
      if (chol_inv32(g, x, lane)) break;
      if (jit) {
        flag |= 2;
        break;
      }
      jit = true;
    }
  }
  st_col<32>(TLi, lane, x);                 // Li rows
  __syncwarp();
  return flag;
}

// ---- 32-token blocks of a [B, T, H, D] tensor <-> a 32 x 32 tile, coalesced ----
// A token row of 32 features is 64 (bf16) or 128 (fp32) contiguous bytes; lanes
// take consecutive 16-byte pieces of consecutive rows, so one warp instruction
// touches 8 (bf16) or 4 (fp32) token rows instead of 32.  Used when every row
// start is 16-byte aligned; otherwise each lane moves its own row.
template <typename IO>
__device__ __forceinline__ bool tok_rows_aligned(const void* p, long long sb, long long st, long long sh, int f0,
                                                 int n) {
  constexpr int kVec = 16 / sizeof(IO);
  return n == 32 && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && sb % kVec == 0 && st % kVec == 0 &&
         sh % kVec == 0 && f0 % kVec == 0;
}

// tile rows [0, 32) <- tokens tok0 + row (rows >= nvalid zero), features [f0, f0 + n)
// the aligned path of load_tok_block in two halves, so that several blocks' loads
// can be in flight together: this lane's 16-byte pieces, then their tile rows
template <typename IO>
struct TokRaw {
  uint4 v[32 / (16 / sizeof(IO))];
};
template <typename IO>
__device__ __forceinline__ void tok_raw_load(TokRaw<IO>& raw, const In& x, int b, int tok0, int h, int f0,
                                             int nvalid, int lane) {
  constexpr int kVec = 16 / sizeof(IO);          // elements per 16-byte piece
  constexpr int kPer = 32 / kVec;                // pieces per token row
  const IO* base = static_cast<const IO*>(x.p) + (long long)b * x.sb + (long long)h * x.sh + f0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int f = 32 * k + lane, row = f / kPer, pc = f % kPer;
    raw.v[k] = __ldg(reinterpret_cast<const uint4*>(base + (long long)(tok0 + (row < nvalid ? row : 0)) * x.st) + pc);
  }
}
template <typename IO>
__device__ __forceinline__ void tok_raw_store(float* Tl, const TokRaw<IO>& raw, int nvalid, int lane) {
  constexpr int kVec = 16 / sizeof(IO);
  constexpr int kPer = 32 / kVec;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int f = 32 * k + lane, row = f / kPer, pc = f % kPer;
    const bool ok = row < nvalid;
    const IO* e = reinterpret_cast<const IO*>(&raw.v[k]);   // registers: plain reads only
    float v[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) v[u] = ok ? to_float(e[u]) : 0.f;
    float4* rowp = reinterpret_cast<float4*>(Tl + row * 32);
#pragma unroll
    for (int c = 0; c < kVec / 4; ++c) {
      const int q = pc * (kVec / 4) + c;       // 16-byte fp32 chunk of the tile row
      rowp[q ^ (row & 7)] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
  }
}

template <typename IO>
__device__ __forceinline__ void load_tok_block(float* Tl, const In& x, int b, int tok0, int h, int f0, int n,
                                               int nvalid, int lane) {
  if (nvalid <= 0) {                             // block past the series end: no loads
    float v[32];
    zero(v);
    st_row(Tl, lane, v);
  } else if (tok_rows_aligned<IO>(x.p, x.sb, x.st, x.sh, f0, n)) {
    TokRaw<IO> raw;
    tok_raw_load<IO>(raw, x, b, tok0, h, f0, nvalid, lane);
    tok_raw_store<IO>(Tl, raw, nvalid, lane);
  } else {
    float v[32];
    ld_tok_row<IO>(v, x, b, tok0 + lane, h, f0, n, lane < nvalid, 1.f);
    st_row(Tl, lane, v);
  }
}

// two consecutive 32-token blocks (tok0, tok0 + 32) into Ta, Tb with both blocks'
// loads in flight together when both are live and aligned
template <typename IO>
__device__ __forceinline__ void load_tok_blocks2(float* Ta, float* Tb, const In& x, int b, int tok0, int h, int f0,
                                                 int n, int nva, int nvb, int lane) {
  if (nva > 0 && nvb > 0 && tok_rows_aligned<IO>(x.p, x.sb, x.st, x.sh, f0, n)) {
    TokRaw<IO> ra, rb;
    tok_raw_load<IO>(ra, x, b, tok0, h, f0, nva, lane);
    tok_raw_load<IO>(rb, x, b, tok0 + 32, h, f0, nvb, lane);
    tok_raw_store<IO>(Ta, ra, nva, lane);
    tok_raw_store<IO>(Tb, rb, nvb, lane);
  } else {
    load_tok_block<IO>(Ta, x, b, tok0, h, f0, n, nva, lane);
    load_tok_block<IO>(Tb, x, b, tok0 + 32, h, f0, n, nvb, lane);
  }
}

// tokens tok0 + row (rows < nvalid), features [f0, f0 + n) <- tile rows
template <typename IO>
__device__ __forceinline__ void store_tok_block(const Out& x, int b, int tok0, int h, int f0, int n, int nvalid,
                                                const float* Tl, int lane) {
  constexpr int kVec = 16 / sizeof(IO);
  constexpr int kPer = 32 / kVec;
  if (tok_rows_aligned<IO>(x.p, x.sb, x.st, x.sh, f0, 32)) {
    IO* base = static_cast<IO*>(x.p) + (long long)b * x.sb + (long long)h * x.sh + f0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int f = 32 * k + lane, row = f / kPer, pc = f % kPer;
      if (row < nvalid && pc * kVec < n) {
        const float4* rowp = reinterpret_cast<const float4*>(Tl + row * 32);
        float v[kVec];
#pragma unroll
        for (int c = 0; c < kVec / 4; ++c) {
          const float4 t = rowp[(pc * (kVec / 4) + c) ^ (row & 7)];
          v[4 * c] = t.x;
          v[4 * c + 1] = t.y;
          v[4 * c + 2] = t.z;
          v[4 * c + 3] = t.w;
        }
        IO* dst = base + (long long)(tok0 + row) * x.st + pc * kVec;
        if constexpr (kVec == 8) {
          __nv_bfloat162 pr[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) pr[u] = __floats2bfloat162_rn(v[2 * u], v[2 * u + 1]);
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(pr);
        } else {
          *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  } else {
    float v[32];
    ld_row(v, Tl, lane);
    st_tok_row<IO>(x, b, tok0 + lane, h, f0, n, lane < nvalid, v, 1.f);
  }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// W / m rows of P block pb (tile TW) as bf16 hi and lo planes in the layout of the
// tensor-core readout operands: the 16-byte row of j-group ng and p sits at byte
// ng * P * 16 + p * 16 of a plane (the lo plane follows the hi plane)
__device__ __forceinline__ void store_wm_block(unsigned char* wq, const float* TW, int pb, int P, int r, int lane) {
  float u[32];
  ld_row(u, TW, lane);
  const int p = pb * 32 + lane;
  if (p >= P) return;
#pragma unroll
  for (int ng = 0; ng < 4; ++ng) {
    if (8 * ng >= r) break;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = u[8 * ng + e];
    uint4 hi, lo;
    split_bf16x8(x, hi, lo);
    *reinterpret_cast<uint4*>(wq + (size_t)ng * P * 16 + (size_t)p * 16) = hi;
    *reinterpret_cast<uint4*>(wq + (size_t)P * r * 2 + (size_t)ng * P * 16 + (size_t)p * 16) = lo;
  }
}

// ops_out: keep the chunk's operators (kOp* tiles) for the backward; wm_out: write
// W / m as the tensor-core readout's operand; nullptr = do not write them.
template <typename IO, int NPB>
__global__ void __launch_bounds__(kMaxWarps * 32) k_fwd_chunk_w(Dims d, In zq, const float* __restrict__ gamma_p,
                                                                Out y, const float* __restrict__ stats,
                                                                const unsigned long long* __restrict__ cmax,
                                                                float* __restrict__ invs_out,
                                                                int* __restrict__ flags_out,
                                                                float* __restrict__ ops_out,
                                                                unsigned char* __restrict__ wm_out) {
  constexpr bool kFast = false;   // fp32-level products (split operands) for every I/O type
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long q = (long long)blockIdx.x * (blockDim.x >> 5) + w;
  if (q >= (long long)d.B * d.H * d.C) return;   // warp-uniform; no block barriers below
  const ChunkId id = chunk_id(d, q);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  extern __shared__ float4 sm4[];
  float* base = reinterpret_cast<float*>(sm4) + (size_t)w * fwd_tiles(P) * kTile;
  float* T0 = base;
  float* T1 = T0 + kTile;
  float* T2 = T1 + kTile;
  float* T3 = T2 + kTile;
  float* TC = T3 + kTile;                   // NPB tiles: Cn rows, later Y blocks
  float* TW = TC + NPB * kTile;             // NPB tiles: (W / m) rows
  const float* rec = stats + q * d.SW;
  // The record's G, M and C rows go out as asynchronous copies into the tiles that
  // hold them first (G -> T0, M -> TW, C -> TC, unscaled), overlapping the series
  // norm and the Cholesky; the 1/m scales move into the products that use them.
  const bool pre = cp_tile_async(T0, rec, r, r, lane);
  cp_async_commit();
  bool pre_mc = pre && cp_tile_async(TW, rec + r * r, r, r, lane);
#pragma unroll
  for (int pb = 0; pb < NPB; ++pb)
    pre_mc = pre_mc && cp_tile_async(TC + pb * kTile, rec + 2 * r * r + pb * 32 * r, P - pb * 32, r, lane);
  cp_async_commit();
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  cp_async_wait<1>();                                                     // G has landed

  const int flag = factor_and_invert(d, rec, lane, im2, false, T0, T1, pre);   // T1 = Li
  if (lane == 0) flags_out[q] = flag;
  float* opq = ops_out ? ops_out + q * (long long)(kNumOps * kOpFloats) : nullptr;
  if (opq) store_op_tile<true>(opq + kOpLi * kOpFloats, T1, lane);   // kept as Li^T
  wmmp<kFast, 32, 32, true, false, false>(T2, T1, kTile, T1, 1.f);        // T2 = S = Li^T Li
  cp_async_wait<0>();                                                     // M and C have landed
  __syncwarp();
  if (opq) store_op_tile<false>(opq + kOpS * kOpFloats, T2, lane);
  const float* TM = TW;                                                   // M (raw): A0 = (M / m^2) S
  if (!pre_mc) {
    load_mat(T0, rec + r * r, r, r, 1.f, lane);
    TM = T0;
  }
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, false>(T3, TM, kTile, T2, im2);       // T3 = A0 = Mn S
  __syncwarp();
  {
    float a[32];
    ld_row(a, T3, lane);
    const float sigma = power_sigma32(a, lane, r);                        // ska.py:41-58
    const float invs = 1.f / fmaxf(sigma, 1.f);
    if (lane == 0) invs_out[q] = invs;
    const float kk = gs * invs;                                           // ska.py:167-169
#pragma unroll
    for (int j = 0; j < 32; ++j) a[j] *= kk;
    __syncwarp();
    st_row(T3, lane, a);                                                  // T3 = A
  }
  __syncwarp();
  if (opq) store_op_tile<false>(opq + kOpA * kOpFloats, T3, lane);
  // A^K (K = 0: identity), ping-pong in T0 / T2
  const float* AK = T3;
  if (d.K == 0) {
    st_identity(T0, lane);
    AK = T0;
  }
  for (int s = 1; s < d.K; ++s) {
    float* out = (AK == T0) ? T2 : T0;
    wmmp<kFast, 32, 32, false, false, false>(out, AK, kTile, T3, 1.f);
    __syncwarp();
    AK = out;
  }
  __syncwarp();
  if (opq) store_op_tile<false>(opq + kOpAK * kOpFloats, AK, lane);
  float* TU = (AK == T0) ? T2 : T0;
  float* TV = (d.K == 1) ? T2 : T3;
  wmmp<kFast, 32, 32, false, false, false>(TU, AK, kTile, T1, 1.f);       // U = A^K Li
  __syncwarp();
  if (opq) store_op_tile<false>(opq + kOpU * kOpFloats, TU, lane);
  wmmp<kFast, 32, 32, true, false, false>(TV, T1, kTile, TU, 1.f);        // V = Li^T U
  if (!pre_mc) {
#pragma unroll
    for (int pb = 0; pb < NPB; ++pb)
      load_mat(TC + pb * kTile, rec + 2 * r * r + pb * 32 * r, P - pb * 32, r, 1.f, lane);   // C rows
  }
  __syncwarp();
  if (opq) store_op_tile<false>(opq + kOpV * kOpFloats, TV, lane);
  wmmp<kFast, 32 * NPB, 32, false, false, false>(TW, TC, kTile, TV, im2);  // W / m = (C / m) V / m
  __syncwarp();
  if (wm_out && (r & 7) == 0) {
    unsigned char* wq = wm_out + (size_t)q * P * r * 4;
#pragma unroll
    for (int pb = 0; pb < NPB; ++pb) store_wm_block(wq, TW + pb * kTile, pb, P, r, lane);
  }
  if (!y.p) return;   // the readout runs as its own tensor-core kernel (k_readout_tc)

  // readout y_t = (W/m) zq_t, 32 tokens per tile: Y block pb = Q (W/m)[pb rows]^T.
  // Two token blocks at a time (T0, T1; Li is dead), both blocks' loads together.
  const int tchunk = id.c * CS;
  for (int t0 = 0; t0 < CS; t0 += 64) {
    const int nva = min(32, min(CS - t0, T - (tchunk + t0)));
    const int nvb = min(32, min(CS - t0 - 32, T - (tchunk + t0 + 32)));
    load_tok_blocks2<IO>(T0, T1, zq, id.b, tchunk + t0, id.h, 0, r, nva, nvb, lane);
    __syncwarp();
    for (int hb = 0; hb < 2 && t0 + 32 * hb < CS; ++hb) {
      const float* TQ = hb ? T1 : T0;
      const int nvalid = hb ? nvb : nva;
#pragma unroll
      for (int pb = 0; pb < NPB; ++pb)
        wmmp<kFast, 32, 32, false, true, false>(TC + pb * kTile, TQ, kTile, TW + pb * kTile, 1.f);
      __syncwarp();
#pragma unroll
      for (int pb = 0; pb < NPB; ++pb)
        store_tok_block<IO>(y, id.b, tchunk + t0 + 32 * hb, id.h, pb * 32, min(32, P - pb * 32), nvalid,
                            TC + pb * kTile, lane);
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
template <typename IO, int NPB>
__global__ void __launch_bounds__(kMaxWarps * 32) k_bwd_chunk_w(Dims d, In zq, In dy,
                                                                const float* __restrict__ gamma_p, Out dzq,
                                                                const float* __restrict__ stats,
                                                                const unsigned long long* __restrict__ cmax,
                                                                const float* __restrict__ invs_in,
                                                                const int* __restrict__ flags_in,
                                                                float* __restrict__ dstats,
                                                                float* __restrict__ dmpart,
                                                                float* __restrict__ dgpart) {
  constexpr bool kFast = false;   // fp32-level products (split operands) for every I/O type
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long q = (long long)blockIdx.x * (blockDim.x >> 5) + w;
  if (q >= (long long)d.B * d.H * d.C) return;
  const ChunkId id = chunk_id(d, q);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  extern __shared__ float4 sm4[];
  float* base = reinterpret_cast<float*>(sm4) + (size_t)w * bwd_tiles(P) * kTile;
  float* TLi = base;
  float* TA = TLi + kTile;
  float* TAK = TA + kTile;
  float* TV = TAK + kTile;
  float* TX = TV + kTile;
  float* TY = TX + kTile;
  float* TW = TY + kTile;                   // NPB tiles: W rows, then dCn rows, then dLi
  float* TDY = TW + NPB * kTile;            // NPB tiles: Cn rows / dY column blocks
  float* TDW = TDY + NPB * kTile;           // NPB tiles: dW rows
  const float* rec = stats + q * d.SW;
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const float gam = *gamma_p;
  const float gs = fminf(fmaxf(gam, 1.f), 1.5f);
  const bool gpass = gam >= 1.f && gam <= 1.5f;       // clamp passes gradients inclusively
  const float kk = gs * invs_in[q];
  const int flag = flags_in[q];
  float t[32], u[32];

  // ---- recompute the forward operator (same arithmetic as k_fwd_chunk_w) ----
  factor_and_invert(d, rec, lane, im2, (flag & 1) != 0, TX, TLi);
  wmmp<kFast, 32, 32, true, false, false>(TY, TLi, kTile, TLi, 1.f);      // TY = S
  ld_gmem_row(t, rec + r * r, lane, r, r, im2);
  st_row(TX, lane, t);                                                    // TX = Mn
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, false>(TA, TX, kTile, TY, 1.f);       // TA = A0
  __syncwarp();
  ld_row(t, TA, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) t[j] *= kk;
  __syncwarp();
  st_row(TA, lane, t);                                                    // TA = A
  __syncwarp();
  const float* AK = TAK;
  if (d.K == 0) {
    st_identity(TAK, lane);
  } else if (d.K == 1) {
    AK = TA;
  } else {
    const float* cur = TA;
    for (int s = 1; s < d.K; ++s) {
      float* out = (s == d.K - 1) ? TAK : ((s & 1) ? TX : TY);
      wmmp<kFast, 32, 32, false, false, false>(out, cur, kTile, TA, 1.f);
      __syncwarp();
      cur = out;
    }
  }
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, false>(TX, AK, kTile, TLi, 1.f);      // TX = U
  __syncwarp();
  wmmp<kFast, 32, 32, true, false, false>(TV, TLi, kTile, TX, 1.f);       // TV = V
#pragma unroll
  for (int pb = 0; pb < NPB; ++pb) {
    ld_gmem_row(t, rec + 2 * r * r, pb * 32 + lane, P, r, im);
    st_row(TDY + pb * kTile, lane, t);                                    // Cn rows
    zero(t);
    st_row(TDW + pb * kTile, lane, t);                                    // dW = 0
  }
  __syncwarp();
  wmmp<kFast, 32 * NPB, 32, false, false, false>(TW, TDY, kTile, TV, 1.f);  // W = Cn V
  __syncwarp();

  // ---- token pass: dW += dY^T qn, dqn = dY W  (32 tokens at a time) ----
  const int tchunk = id.c * CS;
  float dmq = 0.f;
  for (int t0 = 0; t0 < CS; t0 += 32) {
    const int tl = t0 + lane, tok = tchunk + tl;
    const bool live = tl < CS && tok < T;
    ld_tok_row<IO>(u, zq, id.b, tok, id.h, 0, r, live, 1.f);            // zq row (kept for dm)
    st_row(TX, lane, u);
#pragma unroll
    for (int pb = 0; pb < NPB; ++pb) {
      ld_tok_row<IO>(t, dy, id.b, tok, id.h, pb * 32, min(32, P - pb * 32), live, 1.f);
      st_row(TDY + pb * kTile, lane, t);                                  // dY column block pb
    }
    __syncwarp();
    // bf16 dy and zq are exact in tf32: dW needs one product per tile, dqn two
    wmmp<kFast, 32 * NPB, 32, true, false, true>(TDW, TDY, kTile, TX, im);  // dW += dY^T qn
    wmmp<kFast, 32, 32 * NPB, false, false, false>(TY, TDY, kTile, TW, 1.f);         // dqn = dY W
    __syncwarp();
    ld_row(t, TY, lane);
    st_tok_row<IO>(dzq, id.b, tok, id.h, 0, r, live, t, im);             // dzq = dqn / m
    if (live) {
#pragma unroll
      for (int j = 0; j < 32; ++j) dmq = fmaf(t[j], u[j], dmq);   // dqn . zq
    }
    __syncwarp();
  }

  // ---- dV = Cn^T dW,  dCn = dW V^T ----
#pragma unroll
  for (int pb = 0; pb < NPB; ++pb) {
    ld_gmem_row(t, rec + 2 * r * r, pb * 32 + lane, P, r, im);
    st_row(TDY + pb * kTile, lane, t);                                    // Cn rows again
  }
  __syncwarp();
  wmmp<kFast, 32, 32 * NPB, true, false, false>(TX, TDY, kTile, TDW, 1.f);  // TX = dV
  wmmp<kFast, 32 * NPB, 32, false, true, false>(TW, TDW, kTile, TV, 1.f);   // TW = dCn
  __syncwarp();
  float dmc = 0.f;
#pragma unroll
  for (int pb = 0; pb < NPB; ++pb) {
    const int p = pb * 32 + lane;
    ld_row(t, TW + pb * kTile, lane);
    ld_row(u, TDY + pb * kTile, lane);
    if (p < P) {
      float* out = dstats + q * d.SW + 2 * r * r + (size_t)p * r;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < r) {
          out[j] = t[j] * im;
          dmc = fmaf(t[j], u[j], dmc);
        }
      }
    }
  }
  __syncwarp();
  // free now: TW, TDY, TDW, TV ; live: TLi, TA, AK, TX (dV)
  float* TdLi = TW;
  float* TdU = TY;
  float* TU = TDW;
  float* TdAK = TDY;
  wmmp<kFast, 32, 32, false, false, false>(TdU, TLi, kTile, TX, 1.f);      // dU = Li dV
  wmmp<kFast, 32, 32, false, false, false>(TU, AK, kTile, TLi, 1.f);       // U = A^K Li
  __syncwarp();
  wmmp<kFast, 32, 32, false, true, false>(TdLi, TU, kTile, TX, 1.f);       // dLi = U dV^T
  wmmp<kFast, 32, 32, false, true, false>(TdAK, TdU, kTile, TLi, 1.f);     // dAK = dU Li^T
  __syncwarp();
  wmmp<kFast, 32, 32, true, false, true>(TdLi, AK, kTile, TdU, 1.f);       // dLi += AK^T dU
  __syncwarp();
  // dA from dAK; free: TV, TX, TY, TDW
  const float* TdA;
  if (d.K == 0) {
    zero(t);
    st_row(TV, lane, t);
    TdA = TV;
  } else if (d.K == 1) {
    TdA = TdAK;
  } else {
    // Horner over E_s = dAK (A^T)^s:  E <- E A^T,  H <- E + A^T H,  E = H = dAK at start
    float* pool[4] = {TV, TX, TY, TDW};
    const float* E = TdAK;
    const float* Hc = TdAK;
    int pi = 0;
    for (int s = 1; s < d.K; ++s) {
      float* En = pool[pi & 3];
      float* Hn = pool[(pi + 1) & 3];
      pi += 2;
      wmmp<kFast, 32, 32, false, true, false>(En, E, kTile, TA, 1.f);      // E A^T
      __syncwarp();
      ld_row(t, En, lane);
      st_row(Hn, lane, t);
      __syncwarp();
      wmmp<kFast, 32, 32, true, false, true>(Hn, TA, kTile, Hc, 1.f);      // + A^T H
      __syncwarp();
      E = En;
      Hc = Hn;
    }
    TdA = Hc;
  }
  // d gamma: A = gs * invs * A0  ->  d gs = <dA, A> / gs
  float dg = 0.f;
  ld_row(t, TdA, lane);
  ld_row(u, TA, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) dg = fmaf(t[j], u[j], dg);
  // scratch tiles now: three of {TV, TX, TY, TDW, TdAK} not holding dA
  float* fr[3];
  {
    float* cand[5] = {TV, TX, TY, TDW, TdAK};
    int nf = 0;
    for (int i = 0; i < 5 && nf < 3; ++i)
      if (cand[i] != TdA) fr[nf++] = cand[i];
  }
  float* TS = fr[0];
  float* TdMn = fr[1];
  float* TdS = fr[2];
  __syncwarp();
  wmmp<kFast, 32, 32, true, false, false>(TS, TLi, kTile, TLi, 1.f);       // S
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, false>(TdMn, TdA, kTile, TS, kk);      // dMn = kk dA S
  __syncwarp();
  float dmm = 0.f;
  ld_row(t, TdMn, lane);
  ld_gmem_row(u, rec + r * r, lane, r, r, im2);                           // Mn row
  if (lane < r) {
    float* out = dstats + q * d.SW + r * r + (size_t)lane * r;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < r) {
        out[j] = t[j] * im2;
        dmm = fmaf(t[j], u[j], dmm);
      }
    }
  }
  st_row(TS, lane, u);                                                    // TS = Mn (S done)
  __syncwarp();
  wmmp<kFast, 32, 32, true, false, false>(TdS, TS, kTile, TdA, kk);        // dS = kk Mn^T dA
  __syncwarp();
  ld_row(t, TdS, lane);
  ld_col<32>(u, TdS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) t[j] += u[j];                              // (dS + dS^T) row
  st_row(TdMn, lane, t);
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, true>(TdLi, TLi, kTile, TdMn, 1.f);    // dLi += Li (dS + dS^T)
  __syncwarp();
  ld_row(t, TdLi, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j > lane) t[j] = 0.f;                                             // only tril(dLi) reaches L
  st_row(TdLi, lane, t);
  __syncwarp();
  wmmp<kFast, 32, 32, false, true, false>(TS, TdLi, kTile, TLi, -1.f);     // -dLi Li^T
  __syncwarp();
  ld_row(t, TS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j > lane) t[j] = 0.f;                                             // Pm = tril(-dLi Li^T)
  __syncwarp();
  st_row(TS, lane, t);
  __syncwarp();
  ld_col<32>(u, TS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) t[j] = 0.5f * ((j <= lane) ? t[j] : u[j]);   // (Pm + tril(Pm,-1)^T) / 2
  st_row(TdS, lane, t);
  __syncwarp();
  wmmp<kFast, 32, 32, false, false, false>(TdMn, TdS, kTile, TLi, 1.f);    // T1 = P' Li
  __syncwarp();
  wmmp<kFast, 32, 32, true, false, false>(TdS, TLi, kTile, TdMn, 1.f);     // dGn = Li^T T1
  __syncwarp();
  ld_row(t, TdS, lane);
  ld_col<32>(u, TdS, lane);
  float grow[32];
  ld_gmem_row(grow, rec, lane, r, r, 1.f);
  __syncwarp();
  st_row(TS, lane, grow);
  __syncwarp();
  float gcol[32];
  ld_col<32>(gcol, TS, lane);
  float dmg = 0.f;
  if (lane < r) {
    float* out = dstats + q * d.SW + (size_t)lane * r;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < r) {
        const float gsym = 0.5f * (t[j] + u[j]);
        out[j] = gsym * im2;
        dmg = fmaf(gsym, 0.5f * (grow[j] + gcol[j]) * im2, dmg);
      }
    }
  }
  const float tot = warp_sum32(2.f * dmg + 2.f * dmm + dmc + dmq * im);
  const float dgs = warp_sum32(dg);
  if (lane == 0) {
    dmpart[q] = -tot / m;
    dgpart[q] = gpass ? dgs / gs : 0.f;
  }
}


// ---------------------------------------------------------------------------
// backward without the token pass (bf16 token tensors on the tensor-core path),
// from the operators the forward kept
//
// The token-level products live elsewhere: dW' = sum_t dy_t zq_t^T comes from
// k_dw_ps / k_dw_tc, and dzq = dy (W / m) is formed by k_tok_bwd_tc from the
// W / m planes the forward wrote.  The forward also kept the chunk's Li, A, A^K,
// U, V and S (kOp* tiles), so nothing of the forward is recomputed here (no
// Cholesky, no inverse, no power iteration): what remains is the chain rule.
//   dW = dW' / m, dV = Cn^T dW = C^T dW' / m^2, dCn = dW V^T = dW' V^T / m;
// the readout's share of d(max norm) is sum_t dqn_t . zq_t / m = <W, dW> = <V, dV>.
// The P x r blocks of C and dW' stream through two tiles, so a warp holds 8 tiles
// whatever P is.
// ---------------------------------------------------------------------------
constexpr int kBwdStreamTiles = 8;

// tile T <- rows [0, nrows) x columns [0, ncols) of a row-major global matrix, by
// cp.async when the source allows it (then it belongs to the lane's next commit
// group), else by plain loads
__device__ __forceinline__ void fetch_tile(float* T, const float* src, int nrows, int ncols, int lane) {
  if (!cp_tile_async(T, src, nrows, ncols, lane)) load_mat(T, src, nrows, ncols, 1.f, lane);
}

__global__ void __launch_bounds__(kMaxWarps * 32) k_bwd_chunk_s(Dims d, const float* __restrict__ gamma_p,
                                                                const float* __restrict__ stats,
                                                                const unsigned long long* __restrict__ cmax,
                                                                const float* __restrict__ invs_in,
                                                                const float* __restrict__ ops,
                                                                const float* __restrict__ dwraw,
                                                                float* __restrict__ dstats,
                                                                float* __restrict__ dmpart,
                                                                float* __restrict__ dgpart) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long q = (long long)blockIdx.x * (blockDim.x >> 5) + w;
  if (q >= (long long)d.B * d.H * d.C) return;
  const ChunkId id = chunk_id(d, q);
  const int r = d.r, P = d.P;
  extern __shared__ float4 sm4[];
  float* base = reinterpret_cast<float*>(sm4) + (size_t)w * kBwdStreamTiles * kTile;
  float* TLt = base;             // Li^T (the operator is kept transposed)
  float* TA = TLt + kTile;
  float* TAK = TA + kTile;
  float* TV = TAK + kTile;
  float* TX = TV + kTile;       // dV
  float* TY = TX + kTile;
  float* TP0 = TY + kTile;
  float* TP1 = TP0 + kTile;
  const float* rec = stats + q * d.SW;
  const float* opq = ops + q * (long long)(kNumOps * kOpFloats);
  const float* dwq = dwraw + q * (long long)P * r;
  const float* crec = rec + 2 * r * r;
  // group 0: V and the first P block of C and dW'; group 1: Li, A, A^K
  cp_op_async(TV, opq + kOpV * kOpFloats, lane);
  fetch_tile(TP0, crec, min(32, P), r, lane);
  fetch_tile(TP1, dwq, min(32, P), r, lane);
  cp_async_commit();
  cp_op_async(TLt, opq + kOpLi * kOpFloats, lane);
  cp_op_async(TA, opq + kOpA * kOpFloats, lane);
  cp_op_async(TAK, opq + kOpAK * kOpFloats, lane);
  cp_async_commit();
  const float m = series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
  const float gam = *gamma_p;
  const float gs = fminf(fmaxf(gam, 1.f), 1.5f);
  const bool gpass = gam >= 1.f && gam <= 1.5f;       // clamp passes gradients inclusively
  const float kk = gs * invs_in[q];
  float t[32], u[32];

  // ---- P blocks: dV = C^T dW' / m^2,  dCn / m = dW' V^T / m^2 ----
  float dmc = 0.f;
#pragma unroll 1
  for (int pb = 0; pb < p_blocks(P); ++pb) {
    const int p = pb * 32 + lane;
    if (pb > 0) {
      __syncwarp();
      fetch_tile(TP0, crec + pb * 32 * r, P - pb * 32, r, lane);
      fetch_tile(TP1, dwq + pb * 32 * r, P - pb * 32, r, lane);
      cp_async_commit();
      cp_async_wait<0>();
    } else {
      cp_async_wait<1>();
    }
    __syncwarp();
    if (pb == 0)
      wmmp<false, 32, 32, true, false, false>(TX, TP0, kTile, TP1, im2);   // dV  = C^T dW' / m^2
    else
      wmmp<false, 32, 32, true, false, true>(TX, TP0, kTile, TP1, im2);    // dV += C^T dW' / m^2
    wmmp<false, 32, 32, false, true, false>(TY, TP1, kTile, TV, 1.f);      // TY = dW' V^T = m dCn
    __syncwarp();
    ld_row(t, TY, lane);
    ld_row(u, TP0, lane);
    if (p < P) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < r) dmc = fmaf(t[j], u[j], dmc);           // <TY, C> = m^2 <dCn, Cn>
    }
    store_mat(dstats + q * d.SW + 2 * r * r + pb * 32 * r, TY, P - pb * 32, r, im2, lane);   // dCn / m
  }
  __syncwarp();
  float dmq = 0.f;                                        // <V, dV> = <W, dW>
  ld_row(t, TV, lane);
  ld_row(u, TX, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) dmq = fmaf(t[j], u[j], dmq);
  __syncwarp();
  // V is dead: U -> TY, S -> TP1 (group 2)
  cp_op_async(TY, opq + kOpU * kOpFloats, lane);
  cp_op_async(TP1, opq + kOpS * kOpFloats, lane);
  cp_async_commit();
  cp_async_wait<1>();                                     // Li, A, A^K have landed
  __syncwarp();
  // live: TLt, TA, TAK, TX (dV); U, S in flight
  float* TdU = TV;
  float* TdLi = TP0;
  wmmp<false, 32, 32, true, false, false>(TdU, TLt, kTile, TX, 1.f);       // dU = Li dV
  cp_async_wait<0>();
  __syncwarp();
  wmmp<false, 32, 32, false, true, false>(TdLi, TY, kTile, TX, 1.f);       // dLi = U dV^T
  __syncwarp();
  float* TdAK = TX;                                                       // dV is dead
  wmmp<false, 32, 32, false, false, false>(TdAK, TdU, kTile, TLt, 1.f);    // dAK = dU Li^T
  wmmp<false, 32, 32, true, false, true>(TdLi, TAK, kTile, TdU, 1.f);      // dLi += AK^T dU
  __syncwarp();
  // dA from dAK; free: TY (U), TV (dU), TAK
  const float* TdA;
  if (d.K == 0) {
    zero(t);
    st_row(TV, lane, t);
    TdA = TV;
  } else if (d.K == 1) {
    TdA = TdAK;
  } else {
    // Horner over E_s = dAK (A^T)^s:  E <- E A^T,  H <- E + A^T H,  E = H = dAK at start
    float* pool[4] = {TY, TV, TAK, TX};
    const float* E = TdAK;
    const float* Hc = TdAK;
    int pi = 0;
    for (int s = 1; s < d.K; ++s) {
      float* En = pool[pi & 3];
      float* Hn = pool[(pi + 1) & 3];
      pi += 2;
      wmmp<false, 32, 32, false, true, false>(En, E, kTile, TA, 1.f);      // E A^T
      __syncwarp();
      ld_row(t, En, lane);
      st_row(Hn, lane, t);
      __syncwarp();
      wmmp<false, 32, 32, true, false, true>(Hn, TA, kTile, Hc, 1.f);      // + A^T H
      __syncwarp();
      E = En;
      Hc = Hn;
    }
    TdA = Hc;
  }
  float dg = 0.f;
  ld_row(t, TdA, lane);
  ld_row(u, TA, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) dg = fmaf(t[j], u[j], dg);
  // three scratch tiles among {TY, TV, TAK, TX, TA} not holding dA (A is dead now)
  float* fr[3];
  {
    float* cand[5] = {TY, TV, TAK, TX, TA};
    int nf = 0;
    for (int i = 0; i < 5 && nf < 3; ++i)
      if (cand[i] != TdA) fr[nf++] = cand[i];
  }
  float* TS = TP1;
  float* TMn = fr[0];
  float* TdMn = fr[1];
  float* TdS = fr[2];
  __syncwarp();
  wmmp<false, 32, 32, false, false, false>(TdMn, TdA, kTile, TS, kk);      // dMn = kk dA S
  __syncwarp();
  float dmm = 0.f;
  load_mat(TMn, rec + r * r, r, r, im2, lane);                            // Mn
  store_mat(dstats + q * d.SW + r * r, TdMn, r, r, im2, lane);            // dMn / m^2
  __syncwarp();
  ld_row(t, TdMn, lane);
  ld_row(u, TMn, lane);
  if (lane < r) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < r) dmm = fmaf(t[j], u[j], dmm);
  }
  wmmp<false, 32, 32, true, false, false>(TdS, TMn, kTile, TdA, kk);       // dS = kk Mn^T dA
  __syncwarp();
  ld_row(t, TdS, lane);
  ld_col<32>(u, TdS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) t[j] += u[j];                              // (dS + dS^T) row
  st_row(TdMn, lane, t);
  __syncwarp();
  wmmp<false, 32, 32, true, false, true>(TdLi, TLt, kTile, TdMn, 1.f);     // dLi += Li (dS + dS^T)
  __syncwarp();
  ld_row(t, TdLi, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j > lane) t[j] = 0.f;                                             // only tril(dLi) reaches L
  st_row(TdLi, lane, t);
  __syncwarp();
  wmmp<false, 32, 32, false, false, false>(TS, TdLi, kTile, TLt, -1.f);    // -dLi Li^T (S is dead)
  __syncwarp();
  ld_row(t, TS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j > lane) t[j] = 0.f;                                             // Pm = tril(-dLi Li^T)
  __syncwarp();
  st_row(TS, lane, t);
  __syncwarp();
  ld_col<32>(u, TS, lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) t[j] = 0.5f * ((j <= lane) ? t[j] : u[j]);   // (Pm + tril(Pm,-1)^T) / 2
  st_row(TdS, lane, t);
  __syncwarp();
  wmmp<false, 32, 32, false, true, false>(TdMn, TdS, kTile, TLt, 1.f);     // T1 = P' Li
  __syncwarp();
  wmmp<false, 32, 32, false, false, false>(TdS, TLt, kTile, TdMn, 1.f);    // dGn = Li^T T1
  __syncwarp();
  ld_row(t, TdS, lane);
  ld_col<32>(u, TdS, lane);
  __syncwarp();
  load_mat(TS, rec, r, r, 1.f, lane);                                     // TS = G (raw)
  __syncwarp();
  float grow[32], gcol[32];
  ld_row(grow, TS, lane);
  ld_col<32>(gcol, TS, lane);
  float dmg = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float gsym = 0.5f * (t[j] + u[j]);
    if (lane < r && j < r) dmg = fmaf(gsym, 0.5f * (grow[j] + gcol[j]) * im2, dmg);
    t[j] = gsym;
  }
  st_row(TdMn, lane, t);                                                  // T1 is dead: sym(dGn)
  __syncwarp();
  store_mat(dstats + q * d.SW, TdMn, r, r, im2, lane);                    // dGn / m^2
  const float tot = warp_sum32(2.f * dmg + 2.f * dmm + dmc * im2 + dmq);
  const float dgs = warp_sum32(dg);
  if (lane == 0) {
    dmpart[q] = -tot / m;
    dgpart[q] = gpass ? dgs / gs : 0.f;
  }
}
}  // namespace wpc

// ---------------------------------------------------------------------------
// host launch helpers
// ---------------------------------------------------------------------------
bool warp_path_ok(const Dims& d) { return d.r <= 32 && d.P <= 128; }

// Warps (chunks) per CTA: the count that fits the most warps on one SM, given
// 228 KB of shared memory per SM and 1 KB reserved per resident CTA (ties go to
// the larger CTA).  0 when one warp's tiles do not fit.
static int warps_for(size_t per_warp) {
  constexpr size_t kSmPerSm = 228 * 1024, kReserve = 1024;
  int best = 0, best_total = 0;
  for (int nw = wpc::kMaxWarps; nw >= 1; --nw) {
    const size_t cta = (size_t)nw * per_warp;
    if (cta > wpc::kSmemBudget) continue;
    const int total = (int)(kSmPerSm / (cta + kReserve)) * nw;
    if (total > best_total) {
      best_total = total;
      best = nw;
    }
  }
  return best;
}
static size_t fwd_warp_bytes(const Dims& d) { return (size_t)wpc::fwd_tiles(d.P) * wpc::kTile * sizeof(float); }
static size_t bwd_warp_bytes(const Dims& d) { return (size_t)wpc::bwd_tiles(d.P) * wpc::kTile * sizeof(float); }
// bytes for one warp's tiles; 0 when even one warp does not fit
size_t smem_fwd_chunk_w(const Dims& d) { return warps_for(fwd_warp_bytes(d)) > 0 ? fwd_warp_bytes(d) : 0; }
size_t smem_bwd_chunk_w(const Dims& d) { return warps_for(bwd_warp_bytes(d)) > 0 ? bwd_warp_bytes(d) : 0; }

template <typename Kern>
static cudaError_t launch_w(Kern kern, const Dims& d, size_t per_warp, cudaStream_t st, void** args) {
  const int nw = warps_for(per_warp);
  const size_t smem = (size_t)nw * per_warp;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long nq = (long long)d.B * d.H * d.C;
  const unsigned grid = (unsigned)((nq + nw - 1) / nw);
  e = cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(nw * 32), args, smem, st);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename IO>
cudaError_t launch_fwd_chunk_w(const Dims& d, const In& zq, const float* gamma, const Out& y, const float* stats,
                               const unsigned long long* cmax, float* invs, int* flags, float* ops,
                               unsigned char* wm, cudaStream_t st) {
  Dims dd = d;
  In zz = zq;
  Out yy = y;
  void* args[] = {&dd, &zz, (void*)&gamma, &yy, (void*)&stats, (void*)&cmax, (void*)&invs, (void*)&flags,
                  (void*)&ops, (void*)&wm};
  const size_t pw = fwd_warp_bytes(d);
  switch (wpc::p_blocks(d.P)) {
    case 1: return launch_w(wpc::k_fwd_chunk_w<IO, 1>, d, pw, st, args);
    case 2: return launch_w(wpc::k_fwd_chunk_w<IO, 2>, d, pw, st, args);
    case 3: return launch_w(wpc::k_fwd_chunk_w<IO, 3>, d, pw, st, args);
    default: return launch_w(wpc::k_fwd_chunk_w<IO, 4>, d, pw, st, args);
  }
}

template <typename IO>
cudaError_t launch_bwd_chunk_w(const Dims& d, const In& zq, const In& dy, const float* gamma, const Out& dzq,
                               const float* stats, const unsigned long long* cmax, const float* invs,
                               const int* flags, float* dstats, float* dmpart, float* dgpart, cudaStream_t st) {
  Dims dd = d;
  In zz = zq, yy = dy;
  Out oo = dzq;
  void* args[] = {&dd, &zz, &yy, (void*)&gamma, &oo, (void*)&stats, (void*)&cmax, (void*)&invs, (void*)&flags,
                  (void*)&dstats, (void*)&dmpart, (void*)&dgpart};
  const size_t pw = bwd_warp_bytes(d);
  switch (wpc::p_blocks(d.P)) {
    case 1: return launch_w(wpc::k_bwd_chunk_w<IO, 1>, d, pw, st, args);
    case 2: return launch_w(wpc::k_bwd_chunk_w<IO, 2>, d, pw, st, args);
    case 3: return launch_w(wpc::k_bwd_chunk_w<IO, 3>, d, pw, st, args);
    default: return launch_w(wpc::k_bwd_chunk_w<IO, 4>, d, pw, st, args);
  }
}

cudaError_t launch_bwd_chunk_s(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               const float* invs, const float* ops, const float* dwraw, float* dstats,
                               float* dmpart, float* dgpart, cudaStream_t st) {
  Dims dd = d;
  void* args[] = {&dd, (void*)&gamma, (void*)&stats, (void*)&cmax, (void*)&invs, (void*)&ops, (void*)&dwraw,
                  (void*)&dstats, (void*)&dmpart, (void*)&dgpart};
  return launch_w(wpc::k_bwd_chunk_s, d, (size_t)wpc::kBwdStreamTiles * wpc::kTile * sizeof(float), st, args);
}

template cudaError_t launch_fwd_chunk_w<float>(const Dims&, const In&, const float*, const Out&, const float*,
                                               const unsigned long long*, float*, int*, float*, unsigned char*,
                                               cudaStream_t);
template cudaError_t launch_fwd_chunk_w<__nv_bfloat16>(const Dims&, const In&, const float*, const Out&,
                                                       const float*, const unsigned long long*, float*, int*,
                                                       float*, unsigned char*, cudaStream_t);
template cudaError_t launch_bwd_chunk_w<float>(const Dims&, const In&, const In&, const float*, const Out&,
                                               const float*, const unsigned long long*, const float*, const int*,
                                               float*, float*, float*, cudaStream_t);
template cudaError_t launch_bwd_chunk_w<__nv_bfloat16>(const Dims&, const In&, const In&, const float*,
                                                       const Out&, const float*, const unsigned long long*,
                                                       const float*, const int*, float*, float*, float*,
                                                       cudaStream_t);

}  // namespace ska
