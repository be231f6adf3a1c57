// ska_tc.cu -- TMA + tcgen05 token-level SKA kernels (bf16 token tensors).
//
// k_stats_tc: raw per-chunk statistics of one (batch, head, chunk) per CTA
//   G'_c = sum_t z_t z_t^T,  M'_c = sum_t z_{t+1} z_t^T,  C'_c = sum_t v_t z_t^T
// (KLF/koopman_lm/ska.py:96-111: the reference's chunk einsums, the boundary
// transition folded into the chunk that owns z_t) and the chunk's key-norm
// maximum (ska.py:441).  The three products are ONE tensor-core product:
//     [G'; M'; C']  ((2r + P) x r)  =  [Z^T; Z+^T; V^T] (x CS tokens) . Z (CS x r)
// with tokens as K.  TMA writes the three token tiles back to back in the
// canonical no-swizzle layout (ska_tc.cuh), so the stacked A operand is just the
// shared-memory tile read MN-major, and B is its Z part.  bf16 products are exact
// and accumulate in fp32 in TMEM, 128 rows per MMA block.
//
// Every wait is bounded.  A wait that runs out marks the chunk in `status`
// (1: TMA, 2: MMA), waits once more (bounded) for the copies or MMAs in flight,
// poisons the chunk's record with NaN so that it cannot pass silently, frees its
// TMEM and returns.
#include <algorithm>
#include <mutex>

#include <cudaTypedefs.h>

#include "ska_common.cuh"
#include "ska_tc.cuh"
#include "ska_warp.cuh"

namespace ska {
namespace tc {

constexpr int kStatsThreads = 128;     // 4 warps: TMEM lanes 0-127, one row each
constexpr uint32_t kTmemCols = 512;    // TMEM columns per SM

// Two tile layouts.  sw = 0: 16-byte feature groups, no swizzle (ska_tc.cuh).
// sw = 1 (r and P multiples of 32): TMA boxes of 32 features (64-byte token rows)
// in the 64-byte swizzle, one "atom column" of CS rows x 64 B per 32 features; the
// MN-major operand then has LBO = CS * 64 (next 32 features) and SBO = 512 (next
// 8 tokens).  Wider rows halve the L2 -> SM sectors of 16-byte rows.
struct StatsGeom {
  int nb;              // 128-row MMA blocks covering the 2r + P statistic rows
  uint32_t ncols;      // TMEM columns allocated (power of two >= 32)
  uint32_t grp;        // bytes of one feature group (CS x 16 B), or of one atom column (CS x 64 B)
  int sw;              // 1: 64-byte swizzled atom columns
  size_t smem;         // dynamic shared memory
};

__host__ __device__ inline StatsGeom stats_geom(int r, int P, int CS) {
  StatsGeom g{};
  g.nb = (2 * r + P + 127) / 128;
  uint32_t need = (uint32_t)(g.nb * r), c = 32;
  while (c < need) c <<= 1;
  g.ncols = c;
  g.sw = (r % 32 == 0 && P % 32 == 0) ? 1 : 0;
  g.grp = (uint32_t)CS * (g.sw ? 64u : 16u);
  g.smem = (size_t)g.nb * (g.sw ? 4 : 16) * g.grp + 1024;    // + alignment slack (swizzle atoms)
  return g;
}

// s + lo^2 + hi^2 for the two bf16 values packed in w (low half first)
__device__ __forceinline__ float sq2(uint32_t w, float s) {
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xFFFF0000u);
  return fmaf(hi, hi, fmaf(lo, lo, s));
}

__global__ void __launch_bounds__(kStatsThreads, 8) k_stats_tc(const __grid_constant__ CUtensorMap mz,
                                                            const __grid_constant__ CUtensorMap mv, Dims d,
                                                            StatsGeom g, float* __restrict__ stats,
                                                            unsigned long long* __restrict__ cmax,
                                                            int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long red[kStatsThreads / 32];
  unsigned char* tile =
      smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // TMA destinations: 1024-B aligned
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;                                  // (b, h, c), c fastest
  const int c = (int)(q % d.C);
  const long long bh = q / d.C;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const int rows = 2 * r + P;
  const int fpg = g.sw ? 32 : 8;                       // features per group / atom column
  unsigned char* tz = tile;                            // Z   : r/fpg groups
  unsigned char* tzp = tile + (size_t)(r / fpg) * g.grp;     // Z+  : tokens shifted by one
  unsigned char* tv = tile + (size_t)(2 * r / fpg) * g.grp;  // V   : P/fpg groups

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_fence_init();
    tma_prefetch_map(&mz);
    tma_prefetch_map(&mv);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;
  const int t0 = c * CS;

  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (lane == 0) {
      mbar_expect_tx(&bar_load, (uint32_t)rows * (uint32_t)CS * 2u);
      for (int k = 0; k < r / fpg; ++k) {
        tma_load_4d(tz + (size_t)k * g.grp, &mz, &bar_load, fpg * k, h, t0, b);
        tma_load_4d(tzp + (size_t)k * g.grp, &mz, &bar_load, fpg * k, h, t0 + 1, b);
      }
      for (int k = 0; k < P / fpg; ++k) tma_load_4d(tv + (size_t)k * g.grp, &mv, &bar_load, fpg * k, h, t0, b);
    }
    __syncwarp();
  }
  int st = 0;
  if (!__syncthreads_and(mbar_wait(&bar_load, 0, d.wlim))) {
    st = 1;
    mbar_wait(&bar_load, 0, kWaitLimit);                           // let copies in flight land
  }

  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (st == 0 && lane == 0) {
      fence_after_sync();
      const uint32_t id = idesc_bf16(128, r, true, true);
      const uint32_t a0 = smem_u32(tile), b0 = smem_u32(tz);
      for (int mb = 0; mb < g.nb; ++mb)
        for (int ks = 0; ks < CS / 16; ++ks) {
          if (g.sw)   // 16 tokens = two 8-row groups of 512 B; 32 features per atom column
            mma_bf16(tbase + (uint32_t)(mb * r), sdesc_sw(a0 + (uint32_t)mb * 4u * g.grp + 1024u * ks, g.grp, 512u,
                                                          kSwizzle64),
                     sdesc_sw(b0 + 1024u * ks, g.grp, 512u, kSwizzle64), id, ks > 0);
          else
            mma_bf16(tbase + (uint32_t)(mb * r), sdesc(a0 + (uint32_t)mb * 16u * g.grp + 256u * ks, 128u, g.grp),
                     sdesc(b0 + 256u * ks, 128u, g.grp), id, ks > 0);
        }
      mma_commit(&bar_mma);
    }
    __syncwarp();
  }

  // key-norm maximum over the chunk's real tokens, overlapping the MMAs
  unsigned long long key = 0ull;
  if (st == 0) {
    for (int k = tid; k < CS; k += kStatsThreads) {
      const int t = t0 + k;
      if (t >= T) break;
      float s = 0.f;
      // no swizzle: token row k is 16 B in each group; 64-byte swizzle: 64 B in each
      // atom column at (k/8)*512 + (k%8)*64, its 16-byte pieces permuted (summed anyway)
      const int pieces = g.sw ? 4 : 1;
      const size_t roff = g.sw ? (size_t)(k >> 3) * 512 + (size_t)(k & 7) * 64 : (size_t)k * 16;
      for (int gi = 0; gi < r / fpg; ++gi)
        for (int pc = 0; pc < pieces; ++pc) {
          const uint4 u = *reinterpret_cast<const uint4*>(tz + (size_t)gi * g.grp + roff + 16 * pc);
          s = sq2(u.x, s);
          s = sq2(u.y, s);
          s = sq2(u.z, s);
          s = sq2(u.w, s);
        }
      const unsigned long long kk = pack_max(sqrtf(s), t);
      key = kk > key ? kk : key;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(0xffffffffu, key, o);
    key = y > key ? y : key;
  }
  if (lane == 0) red[warp] = key;

  if (st == 0 && !__syncthreads_and(mbar_wait(&bar_mma, 0, d.wlim))) {
    st = 2;
    mbar_wait(&bar_mma, 0, kWaitLimit);                            // let MMAs in flight finish
  }
  __syncthreads();
  fence_after_sync();

  float* rec = stats + q * d.SW;
  if (st == 0) {
    for (int mb = 0; mb < g.nb; ++mb) {
      const int row = mb * 128 + 32 * warp + lane;
      for (int j0 = 0; j0 < r; j0 += 16) {
        float v[16];
        tmem_ld16(tbase + (uint32_t)(mb * r + j0) + ((uint32_t)(32 * warp) << 16), v);
        if (row < rows) {
          float4* dst = reinterpret_cast<float4*>(rec + (size_t)row * r + j0);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        }
      }
    }
  } else {
    for (int i = tid; i < rows * r; i += kStatsThreads) rec[i] = __int_as_float(0x7fc00000);
  }
  if (tid == 0) {
    unsigned long long m = red[0];
    for (int w = 1; w < kStatsThreads / 32; ++w) m = red[w] > m ? red[w] : m;
    cmax[q] = m;
    status[q] = st;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// k_stats_scan_tc: the statistics and their exclusive (decayed) scan in one pass,
// one CTA per (batch, head) series, walking the series' chunks in order
// (ska.py:114-133, adaptive_chunking.py:225-238).  Warp-specialised:
//   warp 0             TMA copies of chunk c into shared stage c % ns;
//   warp 7             the product of chunk c into TMEM buffer c % kScanBufs
//                      (each warp waits together, one lane issues: copies and
//                      products pipeline instead of alternating in one thread);
//   warps 1-4          record rows: warp w reads TMEM lane quarter w % 4 (rows
//                      32 (w % 4) ..), keeps those rows' running prefix in
//                      registers and writes
//                        record c = prefix;  prefix = alpha prefix + chunk c
//                      (alpha = 1: standard) through a per-warp shared tile as
//                      512-byte warp stores;
//   warps 5, 6         the key-norm maximum of the even / odd chunks from the
//                      shared stage (one token per lane).
// The roles meet only at mbarriers: copy landed, product done, TMEM buffer read,
// stage read (by the product and by the key norms).  This replaces k_stats_tc +
// k_scan_fwd (the scan's read and rewrite of every record) when there are enough
// series to occupy the SMs (r = 32, 2r + P <= 128: one 128-row product per chunk).
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 256;
constexpr int kScanStagesMax = 6;
constexpr int kScanBufs = 4;

__global__ void __launch_bounds__(kScanThreads, 1) k_stats_scan_tc(const __grid_constant__ CUtensorMap mz,
                                                                 const __grid_constant__ CUtensorMap mv, Dims d,
                                                                 StatsGeom g, int ns, float* __restrict__ stats,
                                                                 unsigned long long* __restrict__ cmax,
                                                                 int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load[kScanStagesMax], bar_free[kScanStagesMax], bar_mma[kScanBufs], bar_read[kScanBufs];
  __shared__ uint32_t tmem_slot;
  __shared__ int err;
  unsigned char* tiles = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long bh = blockIdx.x;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T, C = d.C;
  const int rows = 2 * r + P;
  const int fpg = g.sw ? 32 : 8;
  const size_t tile_bytes = (size_t)g.nb * (g.sw ? 4 : 16) * g.grp;
  const uint32_t bufcols = (uint32_t)(g.nb * r);      // TMEM columns of one chunk's product
  float* recs = stats + bh * (long long)C * d.SW;

  if (tid == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&bar_load[i], 1);
      mbar_init(&bar_free[i], 2);   // product done + key norms read
    }
    for (int i = 0; i < kScanBufs; ++i) {
      mbar_init(&bar_mma[i], 1);
      mbar_init(&bar_read[i], 4);
    }
    err = 0;
    mbar_fence_init();
    tma_prefetch_map(&mz);
    tma_prefetch_map(&mv);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {
    // ---- copies: the warp waits together, one lane issues ----
    const auto load_chunk = [&](int c) {
      unsigned char* tz = tiles + (size_t)(c % ns) * tile_bytes;
      unsigned char* tzp = tz + (size_t)(r / fpg) * g.grp;
      unsigned char* tv = tz + (size_t)(2 * r / fpg) * g.grp;
      uint64_t* bar = &bar_load[c % ns];
      const int t0 = c * CS;
      mbar_expect_tx(bar, (uint32_t)rows * (uint32_t)CS * 2u);
      for (int k = 0; k < r / fpg; ++k) {
        tma_load_4d(tz + (size_t)k * g.grp, &mz, bar, fpg * k, h, t0, b);
        tma_load_4d(tzp + (size_t)k * g.grp, &mz, bar, fpg * k, h, t0 + 1, b);
      }
      for (int k = 0; k < P / fpg; ++k) tma_load_4d(tv + (size_t)k * g.grp, &mv, bar, fpg * k, h, t0, b);
    };
    int nload = 0;   // chunks copied so far
    bool ok = true;
    for (int c = 0; c < C; ++c) {
      if (c >= ns) {   // chunk c - ns has left the stage (its product is done, its norms read)
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_free[c % ns], (uint32_t)(c / ns - 1) & 1u, d.wlim));
        if (!ok) break;
      }
      if (lane == 0) load_chunk(c);
      __syncwarp();
      nload = c + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every copy has landed before the CTA leaves (bounded; at once when all went well)
      for (int s = 0; s < ns; ++s) {
        int last = -1;
        for (int c = s; c < nload; c += ns) last = c;
        if (last >= 0) mbar_wait(&bar_load[s], (uint32_t)(last / ns) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else if (warp == 7) {
    // ---- products: the warp waits together, one lane issues ----
    const uint32_t id = idesc_bf16(128, r, true, true);
    int nmma = 0;   // chunks multiplied so far
    bool ok = true;
    for (int c = 0; c < C; ++c) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_load[c % ns], (uint32_t)(c / ns) & 1u, d.wlim));
      if (ok && c >= kScanBufs)
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_read[c % kScanBufs], (uint32_t)(c / kScanBufs - 1) & 1u, d.wlim));
      if (!ok) break;
      if (lane == 0) {
        fence_after_sync();
        const uint32_t a0 = smem_u32(tiles + (size_t)(c % ns) * tile_bytes);
        const uint32_t acc = tbase + (uint32_t)(c % kScanBufs) * bufcols;
        for (int mb = 0; mb < g.nb; ++mb)
          for (int ks = 0; ks < CS / 16; ++ks) {
            if (g.sw)
              mma_bf16(acc + (uint32_t)(mb * r),
                       sdesc_sw(a0 + (uint32_t)mb * 4u * g.grp + 1024u * ks, g.grp, 512u, kSwizzle64),
                       sdesc_sw(a0 + 1024u * ks, g.grp, 512u, kSwizzle64), id, ks > 0);
            else
              mma_bf16(acc + (uint32_t)(mb * r), sdesc(a0 + (uint32_t)mb * 16u * g.grp + 256u * ks, 128u, g.grp),
                       sdesc(a0 + 256u * ks, 128u, g.grp), id, ks > 0);
          }
        mma_commit(&bar_mma[c % kScanBufs]);
      }
      __syncwarp();
      nmma = c + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every product has completed before the CTA leaves (bounded)
      for (int s = 0; s < kScanBufs; ++s) {
        int last = -1;
        for (int c = s; c < nmma; c += kScanBufs) last = c;
        if (last >= 0) mbar_wait(&bar_mma[s], (uint32_t)(last / kScanBufs) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else if (warp <= 4) {
    // ---- record rows ----
    const int q = warp & 3;   // TMEM lane quarter this warp may read
    const int row0 = 32 * q, nrow = min(32, rows - row0);
    float* wtile = reinterpret_cast<float*>(tiles + (size_t)ns * tile_bytes) + (warp - 1) * 1024;
    const float alpha = d.decay ? d.alpha : 1.f;
    float pre[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pre[j] = 0.f;
    for (int c = 0; c < C; ++c) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_mma[c % kScanBufs], (uint32_t)(c / kScanBufs) & 1u, d.wlim))) {
        if (lane == 0) atomicExch(&err, 1);
        break;
      }
      fence_after_sync();
      if (warp == 1 && lane == 0) mbar_arrive(&bar_free[c % ns]);   // the product has read the stage
      float v[32], out[32];
      tmem_ld32(tbase + (uint32_t)(c % kScanBufs) * bufcols + ((uint32_t)row0 << 16), v);
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_read[c % kScanBufs]);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        out[j] = pre[j];
        pre[j] = fmaf(alpha, pre[j], v[j]);
      }
      if (nrow > 0) {
        __syncwarp();
        wpc::st_row(wtile, lane, out);
        __syncwarp();
        wpc::store_mat(recs + (long long)c * d.SW + (size_t)row0 * 32, wtile, nrow, 32, 1.f, lane);
      }
    }
  } else if (warp <= 6) {
    // ---- key norms: warp 5 takes the even chunks, warp 6 the odd ones ----
    for (int c = warp - 5; c < C; c += 2) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_load[c % ns], (uint32_t)(c / ns) & 1u, d.wlim))) {
        if (lane == 0) atomicExch(&err, 1);
        break;
      }
      const unsigned char* tz = tiles + (size_t)(c % ns) * tile_bytes;
      const int t0 = c * CS;
      unsigned long long key = 0ull;
      for (int k = lane; k < CS; k += 32) {   // the token's 64-byte row: four 16-byte units
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const size_t off = g.sw ? (size_t)(k >> 3) * 512 + (size_t)(k & 7) * 64 + 16 * u
                                  : (size_t)u * g.grp + (size_t)k * 16;
          const uint4 x = *reinterpret_cast<const uint4*>(tz + off);
          s0 = sq2(x.x, s0);
          s1 = sq2(x.y, s1);
          s2 = sq2(x.z, s2);
          s3 = sq2(x.w, s3);
        }
        const unsigned long long kk = t0 + k < T ? pack_max(sqrtf((s0 + s1) + (s2 + s3)), t0 + k) : 0ull;
        key = kk > key ? kk : key;
      }
      // warp arg-max: largest norm (its bits order like the value), then smallest token
      const uint32_t nb = (uint32_t)(key >> 32), nt = (uint32_t)key;
      const uint32_t mb = __reduce_max_sync(0xffffffffu, nb);
      const uint32_t mt = __reduce_max_sync(0xffffffffu, nb == mb ? nt : 0u);
      if (lane == 0) {
        cmax[bh * C + c] = ((unsigned long long)mb << 32) | mt;
        status[bh * C + c] = 0;
        mbar_arrive(&bar_free[c % ns]);
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (err) {   // poison the series
    const float nan = __int_as_float(0x7fc00000);
    for (long long i = tid; i < (long long)C * d.SW; i += kScanThreads) recs[i] = nan;
    for (int c = tid; c < C; c += kScanThreads) {
      status[bh * C + c] = 1;
      cmax[bh * C + c] = 0ull;   // defined (if meaningless) key norms for the consumers
    }
  }
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// k_dw_tc: raw per-chunk readout gradient  dW'_c = sum_{t in c} dy_t zq_t^T  (P x r)
// for the backward, the token part of d(W qn) (ska.py:180-181 differentiated; the
// 1/m of qn = zq/m is applied by the chunk kernel).  Same structure as k_stats_tc:
// one CTA per chunk, A = dY^T (P rows, tokens as K) and B = ZQ read MN-major from
// the TMA tiles [ZQ | dY], one TMEM-accumulated bf16 product.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kStatsThreads, 8) k_dw_tc(const __grid_constant__ CUtensorMap mzq,
                                                            const __grid_constant__ CUtensorMap mdy, Dims d,
                                                            StatsGeom g, float* __restrict__ dw,
                                                            int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_slot;
  unsigned char* tile = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;
  const int c = (int)(q % d.C);
  const long long bh = q / d.C;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS;
  const int fpg = g.sw ? 32 : 8;                       // features per group / atom column
  unsigned char* tq = tile;                            // ZQ : r/fpg groups
  unsigned char* ty = tile + (size_t)(r / fpg) * g.grp;     // dY : P/fpg groups (+ room for rows P..127)

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_fence_init();
    tma_prefetch_map(&mzq);
    tma_prefetch_map(&mdy);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;
  const int t0 = c * CS;
  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (lane == 0) {
      mbar_expect_tx(&bar_load, (uint32_t)(r + P) * (uint32_t)CS * 2u);
      for (int k = 0; k < r / fpg; ++k) tma_load_4d(tq + (size_t)k * g.grp, &mzq, &bar_load, fpg * k, h, t0, b);
      for (int k = 0; k < P / fpg; ++k) tma_load_4d(ty + (size_t)k * g.grp, &mdy, &bar_load, fpg * k, h, t0, b);
    }
    __syncwarp();
  }
  int st = 0;
  if (!__syncthreads_and(mbar_wait(&bar_load, 0, d.wlim))) {
    st = 1;
    mbar_wait(&bar_load, 0, kWaitLimit);
  }
  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (st == 0 && lane == 0) {
      fence_after_sync();
      const uint32_t id = idesc_bf16(128, r, true, true);
      const uint32_t a0 = smem_u32(ty), b0 = smem_u32(tq);
      for (int ks = 0; ks < CS / 16; ++ks)
        if (g.sw)
          mma_bf16(tbase, sdesc_sw(a0 + 1024u * ks, g.grp, 512u, kSwizzle64),
                   sdesc_sw(b0 + 1024u * ks, g.grp, 512u, kSwizzle64), id, ks > 0);
        else
          mma_bf16(tbase, sdesc(a0 + 256u * ks, 128u, g.grp), sdesc(b0 + 256u * ks, 128u, g.grp), id, ks > 0);
      mma_commit(&bar_mma);
    }
    __syncwarp();
  }
  if (st == 0 && !__syncthreads_and(mbar_wait(&bar_mma, 0, d.wlim))) {
    st = 2;
    mbar_wait(&bar_mma, 0, kWaitLimit);
  }
  __syncthreads();
  fence_after_sync();
  float* rec = dw + q * (long long)P * r;
  const int row = 32 * warp + lane;
  for (int j0 = 0; j0 < r; j0 += 16) {
    float v[16];
    tmem_ld16(tbase + (uint32_t)j0 + ((uint32_t)(32 * warp) << 16), v);
    if (row < P) {
      float4* dst = reinterpret_cast<float4*>(rec + (size_t)row * r + j0);
      const float nan = __int_as_float(0x7fc00000);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        dst[e] = st ? make_float4(nan, nan, nan, nan)
                    : make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    }
  }
  if (tid == 0) status[q] = st;
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// k_tok_bwd_tc: per-token gradients of one chunk from its scanned statistic
// gradients dG, dM, dC (and the previous chunk's dM), KLF/koopman_lm/ska.py:96-133
// differentiated by hand:
//   dz_t = (dG + dG^T) z_t + dM^T z_{t+1} + dM~ z_{t-1} + dC^T v_t
//   dv_t = dC z_t
// where dM~ is the dM of the chunk that owns the transition (t-1 -> t): this
// chunk's, except the previous chunk's for the first token.  Plus the arg-max
// key's share of d(max norm): dz_t* += dm / ||z_t*|| * z_t*  (ska.py:441), and
// the readout's  dzq_t = (W / m)^T dy_t  (ska.py:180-181).
// In matrix form with tokens as M:
//   dZ  (CS x r) = [Z | Z+ | Z- | V] (CS x (3r+P)) . Bz
//   dV  (CS x P) = Z . Bv
//   dZQ (CS x r) = dY (CS x P) . (W / m)
// A is the TMA token tile [Z | Z+ | Z- | V | dY] read K-major.  Bz and Bv are
// built in shared memory from the fp32 gradients (read straight from global
// memory) as bf16 hi + lo pairs (x = hi + lo to ~2^-16 relative); W / m arrives
// already split, in the layout the backward chunk kernel wrote.  Each product
// runs once per half on the tensor cores, accumulating in fp32 in TMEM.  The
// first token's dM fix-up, the arg-max term and the bf16 stores are the
// epilogue.  Requires CS <= 128 (one 64-row MMA block for CS <= 64, else one
// 128-row block; rows past CS are ignored), r in {32, 64}, P % 16 == 0.  An
// M = 64 accumulator puts row i in TMEM lane 32 (i / 16) + i % 16 (checked on
// B200), so each warp's epilogue takes 16 tokens.
// ---------------------------------------------------------------------------
constexpr int kTokThreads = 128;

// Shared-memory plan of k_tok_bwd_tc; every region starts on a 128-byte boundary.
struct TokGeom {
  uint32_t grp;        // bytes of one feature group of the token tile: CS x 16 B
  uint32_t wbytes;     // W / m hi + lo planes: P * r * 4
  uint32_t o_bzh, o_bzl, o_bvh, o_bvl, o_bw, o_corr;   // region offsets
  uint32_t ncols;      // TMEM columns: dZ at [0, r), dV at [r, r + P), dZQ at [r + P, 2r + P)
  size_t smem;
};

__host__ __device__ inline uint32_t up128(uint32_t x) { return (x + 127u) & ~127u; }

__host__ __device__ inline TokGeom tok_geom(int r, int P, int CS) {
  TokGeom g{};
  g.grp = (uint32_t)CS * 16u;
  // token tile: (3r + 2P) / 8 groups, plus room for the ignored rows CS..127
  const uint32_t tile = (uint32_t)((3 * r + 2 * P) / 8) * g.grp + (uint32_t)(128 - CS) * 16u;
  const uint32_t bz = (uint32_t)((3 * r + P) * r) * 2u, bv = (uint32_t)(r * P) * 2u;
  g.wbytes = (uint32_t)(P * r) * 4u;
  g.o_bzh = up128(tile);
  g.o_bzl = up128(g.o_bzh + bz);
  g.o_bvh = up128(g.o_bzl + bz);
  g.o_bvl = up128(g.o_bvh + bv);
  g.o_bw = up128(g.o_bvl + bv);
  g.o_corr = up128(g.o_bw + g.wbytes);
  uint32_t c = 32;
  while (c < (uint32_t)(2 * r + P)) c <<= 1;
  g.ncols = c;
  g.smem = (size_t)g.o_corr + (size_t)r * 4 + 128;   // + alignment slack of the base
  return g;
}

__device__ __forceinline__ void load_row8(const float* src, float (&x)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// operand row `row` (16 bytes) of the hi and lo halves
__device__ __forceinline__ void store_split(unsigned char* hi, unsigned char* lo, int row, const float (&x)[8]) {
  uint4 h, l;
  split_bf16x8(x, h, l);
  *reinterpret_cast<uint4*>(hi + (size_t)row * 16) = h;
  *reinterpret_cast<uint4*>(lo + (size_t)row * 16) = l;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// bf16 element e of a 16-byte token row -> float
__device__ __forceinline__ void ld_row8_s(const float* src, float (&x)[8]) {   // shared memory
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ float bf16_at(const unsigned char* row, int e) {
  const uint16_t u = *reinterpret_cast<const uint16_t*>(row + 2 * e);
  return __uint_as_float((uint32_t)u << 16);
}

// 16 fp32 accumulator columns -> 16 bf16 at dst (32 bytes, 16-byte aligned)
__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, const float (&x)[16]) {
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const __nv_bfloat162 pr = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
    w[e] = *reinterpret_cast<const uint32_t*>(&pr);
  }
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__device__ __forceinline__ __nv_bfloat16* tok_ptr(const Out& o, int b, int t, int h) {
  return static_cast<__nv_bfloat16*>(o.p) + (long long)b * o.sb + (long long)t * o.st + (long long)h * o.sh;
}

// 16 fp32 accumulator columns of token (b, t, h) -> y[j0 .. j0 + 16) as bf16, or as
// fp32 (y32: the bf16-input / fp32-output mode)
__device__ __forceinline__ void store_y16(const Out& y, int b, int t, int h, int j0, const float (&x)[16], bool y32) {
  if (y32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(y.p) + (long long)b * y.sb + (long long)t * y.st +
                                          (long long)h * y.sh + j0);
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = make_float4(x[4 * e], x[4 * e + 1], x[4 * e + 2], x[4 * e + 3]);
  } else {
    store_bf16x16(tok_ptr(y, b, t, h) + j0, x);
  }
}

__global__ void __launch_bounds__(kTokThreads, 2) k_tok_bwd_tc(const __grid_constant__ CUtensorMap mz,
                                                               const __grid_constant__ CUtensorMap mv,
                                                               const __grid_constant__ CUtensorMap mdy, Dims d,
                                                               TokGeom g, const float* __restrict__ dstats,
                                                               const unsigned char* __restrict__ wm,
                                                               const unsigned long long* __restrict__ cmax,
                                                               const float* __restrict__ dm, Out dz, Out dv,
                                                               Out dzq, bool dzq_on, int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load, bar_mma, bar_mmq, bar_rec;
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long s_max;
  unsigned char* base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;                      // (b, h, c), c fastest
  const int c = (int)(q % d.C);
  const long long bh = q / d.C;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const int t0 = c * CS;
  const int rg = r / 8;
  const int mrows = CS <= 64 ? 64 : 128;               // MMA rows: the chunk's tokens, rounded up
  // r = 32, 32 <= P <= 64: the chunk's gradient record (dG, dM: 8 KB; dC: P r 4 B)
  // arrives by bulk copy in the bz-lo and bv regions, and the operands are built
  // from shared memory
  const bool staged = r == 32 && P >= 32 && P <= 64;
  unsigned char* tile = base;                          // [Z | Z+ | Z- | V | dY] feature groups
  unsigned char* bzh = base + g.o_bzh;
  unsigned char* bzl = base + g.o_bzl;
  unsigned char* bvh = base + g.o_bvh;
  unsigned char* bvl = base + g.o_bvl;
  unsigned char* bw = base + g.o_bw;                   // W / m: hi plane, then lo plane
  float* corr = reinterpret_cast<float*>(base + g.o_corr);   // first-token fix-up, r floats
  const size_t zg = (size_t)rg * g.grp;
  const size_t dyg = (size_t)((3 * r + P) / 8) * g.grp;

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_rec, 1);
    mbar_init(&bar_mmq, 1);
    mbar_fence_init();
    tma_prefetch_map(&mz);
    tma_prefetch_map(&mv);
    tma_prefetch_map(&mdy);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (lane == 0) {
      if (staged) {   // the gradient record first: it is what the operand build waits for
        const float* rec = dstats + q * d.SW;
        mbar_expect_tx(&bar_rec, (uint32_t)(2 * r * r + P * r) * 4u);
        bulk_load(bzl, rec, (uint32_t)(2 * r * r) * 4u, &bar_rec);
        bulk_load(bvh, rec + 2 * r * r, (uint32_t)(P * r) * 4u, &bar_rec);
      }
      const uint32_t tok_bytes = (uint32_t)(3 * r + (dzq_on ? 2 : 1) * P) * (uint32_t)CS * 2u;
      mbar_expect_tx(&bar_load, tok_bytes + (dzq_on ? g.wbytes : 0u));
      for (int k = 0; k < rg; ++k) {
        tma_load_4d(tile + (size_t)k * g.grp, &mz, &bar_load, 8 * k, h, t0, b);
        tma_load_4d(tile + zg + (size_t)k * g.grp, &mz, &bar_load, 8 * k, h, t0 + 1, b);
        tma_load_4d(tile + 2 * zg + (size_t)k * g.grp, &mz, &bar_load, 8 * k, h, t0 - 1, b);
      }
      for (int k = 0; k < P / 8; ++k) {
        tma_load_4d(tile + 3 * zg + (size_t)k * g.grp, &mv, &bar_load, 8 * k, h, t0, b);
        if (dzq_on) tma_load_4d(tile + dyg + (size_t)k * g.grp, &mdy, &bar_load, 8 * k, h, t0, b);
      }
      if (dzq_on) bulk_load(bw, wm + (size_t)q * g.wbytes, g.wbytes, &bar_load);
    }
    __syncwarp();
  }

  // Bz = [(dG + dG^T); dM; dM^T; dC] and Bv = dC^T as K-major operands (overlapping
  // the copies): one 16-byte row holds 8 consecutive k for one n, at
  // (k-group * N + n) * 16.  Column reads (x[i][n], i = 8 kg + e) let the 32 lanes
  // take 32 n; row reads (x[n][8 kg ..]) give each lane its own n and k-group.
  const float* dG = dstats + q * d.SW;
  const float* dM = dG + r * r;
  const float* dC = dG + 2 * r * r;
  // series arg-max key: warp 0's first load goes out with the operand loads
  unsigned long long kmx = 0ull;
  if (warp == 0 && lane < d.C) kmx = cmax[bh * d.C + lane];
  int st = 0;
  if (staged) {
    if (!__syncthreads_and(mbar_wait(&bar_rec, 0, d.wlim))) {
      st = 1;
      mbar_wait(&bar_rec, 0, kWaitLimit);
    }
    // every value this thread builds, read from the staged record before any
    // operand row overwrites it
    const float* sG = reinterpret_cast<const float*>(bzl);   // dG [32][32], then dM
    const float* sM = sG + 32 * 32;
    const float* sC = reinterpret_cast<const float*>(bvh);   // dC [P][32]
    const int n1 = tid >> 2, k1 = tid & 3;   // dG + dG^T and dM^T items: n, k-group
    const int k2 = tid >> 5, n2 = tid & 31;  // dM items: k-group, n
    float a[8], bm[8], cm[8], c4[2][8], c5[2][8];
    ld_row8_s(sG + n1 * 32 + k1 * 8, a);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] += sG[(k1 * 8 + e) * 32 + n1];
#pragma unroll
    for (int e = 0; e < 8; ++e) bm[e] = sM[(k2 * 8 + e) * 32 + n2];
    ld_row8_s(sM + n1 * 32 + k1 * 8, cm);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int it = tid + kTokThreads * i;  // < 4P: dC item (k-group it / 32, n it % 32), Bv item (p it / 4, i-group it % 4)
      if (it < 4 * P) {
#pragma unroll
        for (int e = 0; e < 8; ++e) c4[i][e] = sC[((it >> 5) * 8 + e) * 32 + (it & 31)];
        ld_row8_s(sC + (it >> 2) * 32 + (it & 3) * 8, c5[i]);
      }
    }
    __syncthreads();
    store_split(bzh, bzl, k1 * 32 + n1, a);             // k-groups 0 .. 3: dG + dG^T
    store_split(bzh, bzl, (4 + k2) * 32 + n2, bm);      // k-groups 4 .. 7: dM
    store_split(bzh, bzl, (8 + k1) * 32 + n1, cm);      // k-groups 8 .. 11: dM^T
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int it = tid + kTokThreads * i;
      if (it < 4 * P) {
        store_split(bzh, bzl, (12 + (it >> 5)) * 32 + (it & 31), c4[i]);   // k-groups 12 ..: dC
        store_split(bvh, bvl, (it & 3) * P + (it >> 2), c5[i]);            // Bv[p][i] = dC[p][i]
      }
    }
  } else {
    for (int it = tid; it < rg * r; it += kTokThreads) {             // k-groups 0 .. r/8: dG + dG^T
      const int n = it / rg, kg = it % rg;
      float x[8];
      load_row8(dG + n * r + kg * 8, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] += __ldg(dG + (kg * 8 + e) * r + n);
      store_split(bzh, bzl, kg * r + n, x);
    }
    for (int it = tid; it < rg * r; it += kTokThreads) {             // k-groups r/8 .. r/4: dM
      const int kg = it / r, n = it % r;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __ldg(dM + (kg * 8 + e) * r + n);
      store_split(bzh, bzl, (rg + kg) * r + n, x);
    }
    for (int it = tid; it < rg * r; it += kTokThreads) {             // k-groups r/4 .. 3r/8: dM^T
      const int n = it / rg, kg = it % rg;
      float x[8];
      load_row8(dM + n * r + kg * 8, x);
      store_split(bzh, bzl, (2 * rg + kg) * r + n, x);
    }
    for (int it = tid; it < (P / 8) * r; it += kTokThreads) {        // k-groups 3r/8 ..: dC
      const int kg = it / r, n = it % r;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __ldg(dC + (kg * 8 + e) * r + n);
      store_split(bzh, bzl, (3 * rg + kg) * r + n, x);
    }
    for (int it = tid; it < rg * P; it += kTokThreads) {             // Bv[p][i] = dC[p][i]
      const int p = it / rg, ig = it % rg;
      float x[8];
      load_row8(dC + p * r + ig * 8, x);
      store_split(bvh, bvl, ig * P + p, x);
    }
  }
  // series arg-max key (the first 32 chunks' keys were loaded above)
  if (warp == 0) {
    unsigned long long k = kmx;
    for (int i = lane + 32; i < d.C; i += 32) {
      const unsigned long long x = cmax[bh * d.C + i];
      k = x > k ? x : k;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, k, o);
      k = y > k ? y : k;
    }
    if (lane == 0) s_max = k;
  }
  fence_async_smem();                                  // B operands -> tensor-core proxy
  if (!__syncthreads_and(mbar_wait(&bar_load, 0, d.wlim))) {
    st = 1;
    mbar_wait(&bar_load, 0, kWaitLimit);
  }

  // warp 0 issues the dZ product, warp 1 (at the same time) the dV and dZQ products
  // into their own TMEM columns (one thread issues a tcgen05.mma about every 70
  // cycles whatever its shape); each commits to its own barrier
  if (warp < 2) {   // one lane issues; the rest of the warp waits converged
    if (st == 0 && lane == 0) {
      fence_after_sync();
      const uint32_t a0 = smem_u32(tile), ay = smem_u32(tile + dyg);
      // A operand (tokens x features, K-major) for K step ks: 8-feature groups grp apart
      const auto tok_adesc = [&](uint32_t a, int ks) -> uint64_t { return sdesc(a + 2u * g.grp * ks, g.grp, 128u); };
      const uint32_t lbo_z = (uint32_t)rg * 128u, lbo_v = (uint32_t)(P / 8) * 128u;
      const uint32_t idz = idesc_bf16(mrows, r, false, false), idv = idesc_bf16(mrows, P, false, false);
      const uint32_t idq = idesc_bf16(mrows, r, false, true);   // B = W / m, MN-major
      const int kz = (3 * r + P) / 16, kv = r / 16, kq = P / 16;
      for (int part = 0; part < 2; ++part) {
        const uint32_t bz0 = smem_u32(part ? bzl : bzh), bv0 = smem_u32(part ? bvl : bvh);
        const uint32_t bw0 = smem_u32(bw) + (part ? (uint32_t)(P * r * 2) : 0u);
        if (warp == 0) {
          for (int ks = 0; ks < kz; ++ks)
            mma_bf16(tbase, tok_adesc(a0, ks), sdesc(bz0 + 2u * lbo_z * ks, lbo_z, 128u), idz, part > 0 || ks > 0);
        } else {
          for (int ks = 0; ks < kv; ++ks)
            mma_bf16(tbase + (uint32_t)r, tok_adesc(a0, ks), sdesc(bv0 + 2u * lbo_v * ks, lbo_v, 128u), idv,
                     part > 0 || ks > 0);
          // W / m MN-major: k-groups (8 p) 128 B apart, n-groups (8 j) P * 16 B apart
          for (int ks = 0; dzq_on && ks < kq; ++ks)
            mma_bf16(tbase + (uint32_t)(r + P), tok_adesc(ay, ks), sdesc(bw0 + 256u * ks, 128u, (uint32_t)P * 16u),
                     idq, part > 0 || ks > 0);
        }
      }
      mma_commit(warp == 0 ? &bar_mma : &bar_mmq);
    }
    __syncwarp();
  }
  // first token of a chunk: (dM_prev - dM) z_{t-1}, z_{t-1} = row 0 of Z-; one warp per row
  if (st == 0 && c > 0 && r == 32) {
    // r = 32: lane j holds column j of rows warp + 4u; all 16 loads go out together
    const float* mprev = dM - d.SW;
    const float zj = bf16_at(tile + 2 * zg + (size_t)(lane / 8) * g.grp, lane % 8);
    float dd[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = warp + 4 * u;
      dd[u] = __ldg(mprev + i * 32 + lane) - __ldg(dM + i * 32 + lane);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float a = dd[u] * zj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) corr[warp + 4 * u] = a;
    }
  } else if (st == 0 && c > 0) {
    const unsigned char* zm = tile + 2 * zg;
    const float* mprev = dM - d.SW;
    for (int i = warp; i < r; i += kTokThreads / 32) {
      float a = 0.f;
      for (int j = lane; j < r; j += 32)
        a = fmaf(__ldg(mprev + i * r + j) - __ldg(dM + i * r + j),
                 bf16_at(zm + (size_t)(j / 8) * g.grp, j % 8), a);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) corr[i] = a;
    }
  }
  if (st == 0 && !__syncthreads_and(mbar_wait(&bar_mma, 0, d.wlim) && mbar_wait(&bar_mmq, 0, d.wlim))) {
    st = 2;
    mbar_wait(&bar_mma, 0, kWaitLimit);
    mbar_wait(&bar_mmq, 0, kWaitLimit);
  }
  __syncthreads();
  fence_after_sync();

  // epilogue: token row m sits in TMEM lane 32 warp + lane (M = 128: m = 32 warp + lane)
  // or 32 warp + (m % 16) (M = 64: m = 16 warp + lane for lanes 0-15)
  const int m = mrows == 64 ? 16 * warp + lane : 32 * warp + lane, t = t0 + m;
  const bool live = (mrows == 128 || lane < 16) && m < CS && t < T;
  const unsigned long long kmax = s_max;
  const float raw = unpack_norm(kmax);
  const int tstar = unpack_t(kmax);
  const float arg = (raw >= kNormClamp && raw > 0.f && t == tstar) ? dm[bh] / raw : 0.f;
  const bool first = (m == 0 && c > 0);
  const float nan = __int_as_float(0x7fc00000);
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  for (int j0 = 0; j0 < r; j0 += 16) {                 // dz
    float x[16];
    tmem_ld16(tbase + lane_base + (uint32_t)j0, x);
    if (live) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = j0 + e;
        float a = x[e];
        if (first) a += corr[j];
        if (arg != 0.f) a = fmaf(arg, bf16_at(tile + (size_t)(j / 8) * g.grp + (size_t)m * 16, j % 8), a);
        x[e] = st ? nan : a;
      }
      store_bf16x16(tok_ptr(dz, b, t, h) + j0, x);
    }
  }
  for (int j0 = 0; j0 < P; j0 += 16) {                 // dv
    float x[16];
    tmem_ld16(tbase + lane_base + (uint32_t)(r + j0), x);
    if (live) {
      if (st) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = nan;
      }
      store_bf16x16(tok_ptr(dv, b, t, h) + j0, x);
    }
  }
  for (int j0 = 0; dzq_on && j0 < r; j0 += 16) {      // dzq
    float x[16];
    tmem_ld16(tbase + lane_base + (uint32_t)(r + P + j0), x);
    if (live) {
      if (st) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = nan;
      }
      store_bf16x16(tok_ptr(dzq, b, t, h) + j0, x);
    }
  }
  if (tid == 0) status[q] |= st << 2;   // bits 2-3 (bits 0-1: the readout-gradient kernel)
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static bool stride_ok(long long s_elems, long long extent) {
  return extent == 1 || (s_elems > 0 && (s_elems * 2) % 16 == 0 && s_elems * 2 < (1ll << 40));
}

// A [B, T, H, D] bf16 tensor as a TMA map {D, H, T, B} (the dimension order of
// increasing stride for the usual layouts); box {8, 1, CS, 1}: one feature group
// of CS tokens of one head (16-byte rows), i.e. one column of canonical core
// matrices.  Tokens outside [0, T) read as zeros.
static bool token_map(CUtensorMap* m, const In& x, int B, int T, int H, int D, int CS, bool sw64 = false) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  const auto sub = [](long long s, long long extent) -> cuuint64_t {
    return (cuuint64_t)(extent == 1 ? 16 : s * 2);   // any valid stride for a unit dimension
  };
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {sub(x.sh, H), sub(x.st, T), sub(x.sb, B)};
  cuuint32_t box[4] = {sw64 ? 32u : 8u, 1, (cuuint32_t)CS, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(x.p), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool stats_tc_ok(const Dims& d, const In& z, const In& v) {
  // r % 16: products of N = r columns and 16-column epilogues (r % 32 also takes the
  // 64-byte swizzled tiles when P % 32 == 0, else 16-byte feature groups)
  if (d.r % 16 != 0 || d.r > 64 || d.P % 8 != 0 || d.P > 128 || d.CS % 16 != 0 || d.CS > 256) return false;
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(z.p) || !al(v.p)) return false;
  return stride_ok(z.st, d.T) && stride_ok(z.sh, d.H) && stride_ok(z.sb, d.B) && stride_ok(v.st, d.T) &&
         stride_ok(v.sh, d.H) && stride_ok(v.sb, d.B);
}

size_t stats_tc_smem(const Dims& d) { return stats_geom(d.r, d.P, d.CS).smem; }

// Resident CTAs per SM are capped so that their TMEM allocations always fit at
// once: when the thread limit allows more CTAs than TMEM does, the shared-memory
// request is raised until one more CTA no longer fits in the SM's 228 KB.
static size_t tmem_safe_smem(uint32_t ncols, int threads, size_t smem) {
  const uint32_t tmem_ctas = kTmemCols / ncols;             // >= 1
  const uint32_t thread_ctas = 2048u / (uint32_t)threads;
  if (tmem_ctas >= thread_ctas) return smem;
  const size_t need = (228u * 1024u) / (tmem_ctas + 1) + 1;
  return smem < need ? need : smem;
}

// dzq_on: also dzq = dY (W / m) (needs dy and dzq; W / m from k_bwd_chunk_s)
bool tok_bwd_tc_ok(const Dims& d, const In& z, const In& v, const In& dy, const Out& dz, const Out& dv,
                   const Out& dzq, bool dzq_on) {
  if (!stats_tc_ok(d, z, v) || d.CS > 128 || d.P % 16 != 0) return false;
  if (dzq_on && !stats_tc_ok(d, z, dy)) return false;
  if (tok_geom(d.r, d.P, d.CS).smem > 227u * 1024u - 64u) return false;   // 64 B of static barriers
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const auto s8 = [](long long s, long long extent) { return extent == 1 || s % 8 == 0; };
  const auto out_ok = [&](const Out& o) {   // 16-byte vector stores of token rows
    return al(o.p) && s8(o.st, d.T) && s8(o.sh, d.H) && s8(o.sb, d.B);
  };
  return out_ok(dz) && out_ok(dv) && (!dzq_on || out_ok(dzq));
}

cudaError_t launch_tok_bwd_tc(const Dims& d, const In& z, const In& v, const In& dy, const float* dstats,
                              const unsigned char* wm, const unsigned long long* cmax, const float* dm,
                              const Out& dz, const Out& dv, const Out& dzq, bool dzq_on, int* status,
                              cudaStream_t st) {
  CUtensorMap mz, mv, my;
  const TokGeom g = tok_geom(d.r, d.P, d.CS);
  if (!token_map(&mz, z, d.B, d.T, d.H, d.r, d.CS) || !token_map(&mv, v, d.B, d.T, d.H, d.P, d.CS))
    return cudaErrorInvalidValue;
  if (dzq_on ? !token_map(&my, dy, d.B, d.T, d.H, d.P, d.CS) : !token_map(&my, v, d.B, d.T, d.H, d.P, d.CS))
    return cudaErrorInvalidValue;
  const size_t smem = tmem_safe_smem(g.ncols, kTokThreads, g.smem);
  cudaError_t e = cudaFuncSetAttribute(k_tok_bwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H * d.C;
  k_tok_bwd_tc<<<(unsigned)n, kTokThreads, smem, st>>>(mz, mv, my, d, g, dstats, wm, cmax, dm, dz, dv, dzq, dzq_on,
                                                         status);
  return cudaGetLastError();
}

// dW' needs the A block (P rows) inside one 128-row MMA
// ---------------------------------------------------------------------------
// k_dw_ps: the dW' products of many chunks per CTA (r = 32, P = 64, 64-byte
// swizzled tiles), so that the one-chunk CTAs of k_dw_tc do not leave a partial
// second wave and each CTA's set-up is paid once:
//   warp 0      TMA copies of chunk j's [ZQ | dY] tiles into shared stage j % ns;
//   warp 1      chunk j's M = 64 product dY^T ZQ into TMEM buffer j % kDwBufs;
//   warps 2-5   the epilogue: warp w reads TMEM lane quarter w % 4, whose lanes
//               0-15 hold product rows 16 (w % 4) .. + 15, and writes them as the
//               chunk's fp32 record.
// Each warp waits together and one lane issues; the roles meet only at mbarriers.
// The CTA takes chunks blockIdx.x, blockIdx.x + gridDim.x, ...
// ---------------------------------------------------------------------------
constexpr int kDwThreads = 192;
constexpr int kDwStagesMax = 6;
constexpr int kDwBufs = 4;

__global__ void __launch_bounds__(kDwThreads, 1) k_dw_ps(const __grid_constant__ CUtensorMap mzq,
                                                        const __grid_constant__ CUtensorMap mdy, Dims d,
                                                        uint32_t grp, int ns, float* __restrict__ dw,
                                                        int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load[kDwStagesMax], bar_free[kDwStagesMax], bar_mma[kDwBufs], bar_read[kDwBufs];
  __shared__ uint32_t tmem_slot;
  __shared__ int err;
  unsigned char* tiles = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = d.r, P = d.P, CS = d.CS;
  const long long nq = (long long)d.B * d.H * d.C;
  const int nj = (int)((nq - (long long)blockIdx.x + gridDim.x - 1) / gridDim.x);   // this CTA's chunks
  const size_t stage_bytes = (size_t)(r / 32 + P / 32) * grp;   // ZQ atom column, then the dY ones
  const auto chunk_of = [&](int j) { return (long long)blockIdx.x + (long long)j * gridDim.x; };

  if (tid == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&bar_load[i], 1);
      mbar_init(&bar_free[i], 1);
    }
    for (int i = 0; i < kDwBufs; ++i) {
      mbar_init(&bar_mma[i], 1);
      mbar_init(&bar_read[i], 4);
    }
    err = 0;
    mbar_fence_init();
    tma_prefetch_map(&mzq);
    tma_prefetch_map(&mdy);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, kDwBufs * 32);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {
    // ---- copies ----
    int nload = 0;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      if (j >= ns) {   // chunk j - ns's product has read the stage
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_free[j % ns], (uint32_t)(j / ns - 1) & 1u, d.wlim));
        if (!ok) break;
      }
      if (lane == 0) {
        const long long q = chunk_of(j);
        const int c = (int)(q % d.C);
        const long long bh = q / d.C;
        const int h = (int)(bh % d.H), b = (int)(bh / d.H);
        unsigned char* tq = tiles + (size_t)(j % ns) * stage_bytes;
        unsigned char* ty = tq + (size_t)(r / 32) * grp;
        uint64_t* bar = &bar_load[j % ns];
        mbar_expect_tx(bar, (uint32_t)(r + P) * (uint32_t)CS * 2u);
        for (int k = 0; k < r / 32; ++k) tma_load_4d(tq + (size_t)k * grp, &mzq, bar, 32 * k, h, c * CS, b);
        for (int k = 0; k < P / 32; ++k) tma_load_4d(ty + (size_t)k * grp, &mdy, bar, 32 * k, h, c * CS, b);
      }
      __syncwarp();
      nload = j + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every copy has landed before the CTA leaves (bounded)
      for (int s = 0; s < ns; ++s) {
        int last = -1;
        for (int j = s; j < nload; j += ns) last = j;
        if (last >= 0) mbar_wait(&bar_load[s], (uint32_t)(last / ns) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- products ----
    const uint32_t id = idesc_bf16(64, r, true, true);
    int nmma = 0;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_load[j % ns], (uint32_t)(j / ns) & 1u, d.wlim));
      if (ok && j >= kDwBufs)
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_read[j % kDwBufs], (uint32_t)(j / kDwBufs - 1) & 1u, d.wlim));
      if (!ok) break;
      if (lane == 0) {
        fence_after_sync();
        const uint32_t b0 = smem_u32(tiles + (size_t)(j % ns) * stage_bytes);
        const uint32_t a0 = b0 + (uint32_t)(r / 32) * grp;
        const uint32_t acc = tbase + (uint32_t)(j % kDwBufs) * 32u;
        for (int ks = 0; ks < CS / 16; ++ks)
          mma_bf16(acc, sdesc_sw(a0 + 1024u * ks, grp, 512u, kSwizzle64), sdesc_sw(b0 + 1024u * ks, grp, 512u, kSwizzle64),
                   id, ks > 0);
        mma_commit(&bar_mma[j % kDwBufs]);
      }
      __syncwarp();
      nmma = j + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every product has completed before the CTA leaves (bounded)
      for (int s = 0; s < kDwBufs; ++s) {
        int last = -1;
        for (int j = s; j < nmma; j += kDwBufs) last = j;
        if (last >= 0) mbar_wait(&bar_mma[s], (uint32_t)(last / kDwBufs) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: rows 16 qd + lane (lanes 0-15) of each product ----
    const int qd = warp & 3;
    const int row = 16 * qd + lane;
    for (int j = 0; j < nj; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_mma[j % kDwBufs], (uint32_t)(j / kDwBufs) & 1u, d.wlim))) {
        if (lane == 0) atomicExch(&err, 1);
        break;
      }
      fence_after_sync();
      if (warp == 2 && lane == 0) mbar_arrive(&bar_free[j % ns]);   // the product has read the stage
      float v0[16], v1[16];
      const uint32_t ta = tbase + (uint32_t)(j % kDwBufs) * 32u + ((uint32_t)(32 * qd) << 16);
      tmem_ld16(ta, v0);
      tmem_ld16(ta + 16u, v1);
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_read[j % kDwBufs]);
      const long long q = chunk_of(j);
      if (lane < 16 && row < P) {
        float4* dst = reinterpret_cast<float4*>(dw + q * (long long)P * r + (size_t)row * r);
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = make_float4(v0[4 * e], v0[4 * e + 1], v0[4 * e + 2], v0[4 * e + 3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[4 + e] = make_float4(v1[4 * e], v1[4 * e + 1], v1[4 * e + 2], v1[4 * e + 3]);
      }
      if (warp == 2 && lane == 0) status[q] = 0;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (err) {   // poison this CTA's chunks
    const float nan = __int_as_float(0x7fc00000);
    for (int j = 0; j < nj; ++j) {
      const long long q = chunk_of(j);
      for (int i = tid; i < P * r; i += kDwThreads) dw[q * (long long)P * r + i] = nan;
      if (tid == 0) status[q] = 1;
    }
  }
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, kDwBufs * 32);
  }
}

bool dw_tc_ok(const Dims& d, const In& zq, const In& dy) { return d.P <= 128 && stats_tc_ok(d, zq, dy); }

cudaError_t launch_dw_tc(const Dims& d, const In& zq, const In& dy, float* dw, int* status, cudaStream_t st) {
  CUtensorMap mq, my;
  StatsGeom g = stats_geom(d.r, d.P, d.CS);
  if (!token_map(&mq, zq, d.B, d.T, d.H, d.r, d.CS, g.sw) || !token_map(&my, dy, d.B, d.T, d.H, d.P, d.CS, g.sw))
    return cudaErrorInvalidValue;
  if (g.sw && d.r == 32 && d.P == 64) {   // persistent CTAs, two per SM
    const size_t stage = (size_t)(d.r / 32 + d.P / 32) * g.grp;
    const int ns = (int)std::min<size_t>(kDwStagesMax, (100u * 1024u - 1024u) / stage);
    if (ns >= 2) {
      const size_t smem = (size_t)ns * stage + 1024;
      cudaError_t e = cudaFuncSetAttribute(k_dw_ps, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      int dev = 0, sms = 0;
      if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
      const long long n = (long long)d.B * d.H * d.C;
      const unsigned grid = (unsigned)std::min<long long>(n, 2LL * sms);
      k_dw_ps<<<grid, kDwThreads, smem, st>>>(mq, my, d, g.grp, ns, dw, status);
      return cudaGetLastError();
    }
  }
  g.nb = 1;
  // tcgen05.alloc takes a power of two >= 32 columns (r = 48 takes 64)
  g.ncols = 32u;
  while (g.ncols < (uint32_t)d.r) g.ncols <<= 1;
  // ZQ groups + the groups of 128 A rows (P real)
  g.smem = g.sw ? (size_t)(d.r / 32 + 4) * g.grp + 1024 : (size_t)(d.r / 8 + 16) * g.grp + 1024;
  const size_t smem = tmem_safe_smem(g.ncols, kStatsThreads, g.smem);
  cudaError_t e = cudaFuncSetAttribute(k_dw_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H * d.C;
  k_dw_tc<<<(unsigned)n, kStatsThreads, smem, st>>>(mq, my, d, g, dw, status);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// k_readout_tc: the forward readout  y_t = (W / m) zq_t  of one chunk per CTA
// (KLF/koopman_lm/ska.py:179-186: y = B_v L A^K L^{-1} qn, which is (W / m) zq with
// W = Cn Li^T A^K Li kept by the chunk-operator kernel).  With tokens as M:
//   Y (CS x P) = ZQ (CS x r) . (W / m)^T
// A is the TMA token tile of zq read K-major (features as K); B is W / m as the
// bf16 hi and lo planes the chunk-operator kernel wrote, whose 16-byte rows (8
// consecutive j for one p) are exactly a K-major B operand with N = P, K = r.  The
// bf16 tokens are exact, W / m = hi + lo to ~2^-17, so two products accumulated
// in fp32 in TMEM give y to fp32 level.  Waits are bounded as in the other kernels;
// an expired wait ORs its code into bits 2-3 of the chunk's forward status and
// writes NaN into the chunk's y.
// ---------------------------------------------------------------------------
constexpr int kReadThreads = 128;

struct ReadGeom {
  uint32_t grp;        // bytes of one 8-feature group of the zq tile: CS x 16 B
  uint32_t o_w;        // offset of the W / m planes (after the tile and the M - CS spare rows)
  uint32_t wbytes;     // P * r * 4
  uint32_t ncols;      // TMEM columns: P, rounded up to a power of two >= 32
  int mrows;           // MMA rows: 64 for CS <= 64, else 128
  size_t smem;
};

__host__ __device__ inline ReadGeom read_geom(int r, int P, int CS) {
  ReadGeom g{};
  g.mrows = CS <= 64 ? 64 : 128;
  g.grp = (uint32_t)CS * 16u;
  const uint32_t tile = (uint32_t)(r / 8) * g.grp + (uint32_t)(g.mrows - CS) * 16u;
  g.o_w = up128(tile);
  g.wbytes = (uint32_t)(P * r) * 4u;
  uint32_t c = 32;
  while (c < (uint32_t)P) c <<= 1;
  g.ncols = c;
  g.smem = (size_t)g.o_w + g.wbytes + 128;
  return g;
}

__global__ void __launch_bounds__(kReadThreads) k_readout_tc(const __grid_constant__ CUtensorMap mzq, Dims d,
                                                             ReadGeom g, const unsigned char* __restrict__ wm,
                                                             Out y, bool y32, int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_slot;
  unsigned char* base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;                      // (b, h, c), c fastest
  const int c = (int)(q % d.C);
  const long long bh = q / d.C;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const int t0 = c * CS;
  unsigned char* tile = base;
  unsigned char* bw = base + g.o_w;

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_fence_init();
    tma_prefetch_map(&mzq);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {   // one lane issues; the rest of the warp waits converged
    if (lane == 0) {
      mbar_expect_tx(&bar_load, (uint32_t)r * (uint32_t)CS * 2u + g.wbytes);
      for (int k = 0; k < r / 8; ++k) tma_load_4d(tile + (size_t)k * g.grp, &mzq, &bar_load, 8 * k, h, t0, b);
      bulk_load(bw, wm + (size_t)q * g.wbytes, g.wbytes, &bar_load);
    }
    __syncwarp();
  }
  int st = 0;
  if (!__syncthreads_and(mbar_wait(&bar_load, 0, d.wlim))) {
    st = 1;
    mbar_wait(&bar_load, 0, kWaitLimit);               // let copies in flight land
  }
  if (warp == 0) {
    if (st == 0 && lane == 0) {
      fence_after_sync();
      const uint32_t a0 = smem_u32(tile), b0 = smem_u32(bw);
      const uint32_t id = idesc_bf16(g.mrows, P, false, false);
      const uint32_t lbo_b = (uint32_t)P * 16u;         // next 8 j of W / m
      for (int part = 0; part < 2; ++part)
        for (int ks = 0; ks < r / 16; ++ks)
          mma_bf16(tbase, sdesc(a0 + 2u * g.grp * ks, g.grp, 128u),
                   sdesc(b0 + (uint32_t)part * (uint32_t)(P * r * 2) + 2u * lbo_b * ks, lbo_b, 128u), id,
                   part > 0 || ks > 0);
      mma_commit(&bar_mma);
    }
    __syncwarp();
  }
  if (st == 0 && !__syncthreads_and(mbar_wait(&bar_mma, 0, d.wlim))) {
    st = 2;
    mbar_wait(&bar_mma, 0, kWaitLimit);                // let the products finish
  }
  __syncthreads();
  fence_after_sync();
  // token row m in TMEM lane 32 warp + lane (M = 128) or 32 warp + m % 16 (M = 64, lanes 0-15)
  const int m = g.mrows == 64 ? 16 * warp + lane : 32 * warp + lane, t = t0 + m;
  const bool live = (g.mrows == 128 || lane < 16) && m < CS && t < T;
  const float nan = __int_as_float(0x7fc00000);
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  for (int j0 = 0; j0 < P; j0 += 16) {
    float x[16];
    tmem_ld16(tbase + lane_base + (uint32_t)j0, x);
    if (live) {
      if (st) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = nan;
      }
      store_y16(y, b, t, h, j0, x, y32);
    }
  }
  if (tid == 0 && st) status[q] |= st << 2;            // bits 2-3 (bits 0-1: the statistics kernel)
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// k_readout_ps: the same readout, many chunks per CTA (persistent, two CTAs per
// SM), so that one chunk's copies overlap the previous chunks' products and
// stores:
//   warp 0      TMA copy of chunk j's zq tile and bulk copy of its W / m planes
//               into shared stage j % ns;
//   warp 1      chunk j's products into TMEM buffer j % kReadBufs;
//   warps 2-5   the epilogue: warp w reads TMEM lane quarter w % 4 (rows
//               32 (w % 4) + lane for M = 128, rows 16 (w % 4) + lane of lanes 0-15
//               for M = 64) and stores the chunk's y rows as bf16.
// Each warp waits together and one lane issues; the roles meet only at mbarriers.
// The CTA takes chunks blockIdx.x, blockIdx.x + gridDim.x, ...
// ---------------------------------------------------------------------------
constexpr int kReadPsThreads = 192;
constexpr int kReadStagesMax = 6;
constexpr int kReadBufs = 4;

__global__ void __launch_bounds__(kReadPsThreads, 1) k_readout_ps(const __grid_constant__ CUtensorMap mzq, Dims d,
                                                                  ReadGeom g, uint32_t stage_bytes, int ns,
                                                                  const unsigned char* __restrict__ wm, Out y,
                                                                  bool y32, int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load[kReadStagesMax], bar_free[kReadStagesMax], bar_mma[kReadBufs], bar_read[kReadBufs];
  __shared__ uint32_t tmem_slot;
  __shared__ int err;
  unsigned char* stages = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const long long nq = (long long)d.B * d.H * d.C;
  const int nj = (int)((nq - (long long)blockIdx.x + gridDim.x - 1) / gridDim.x);   // this CTA's chunks
  const auto chunk_of = [&](int j) { return (long long)blockIdx.x + (long long)j * gridDim.x; };

  if (tid == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&bar_load[i], 1);
      mbar_init(&bar_free[i], 1);
    }
    for (int i = 0; i < kReadBufs; ++i) {
      mbar_init(&bar_mma[i], 1);
      mbar_init(&bar_read[i], 4);
    }
    err = 0;
    mbar_fence_init();
    tma_prefetch_map(&mzq);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, kReadBufs * g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {
    // ---- copies ----
    int nload = 0;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      if (j >= ns) {   // chunk j - ns's products have read the stage
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_free[j % ns], (uint32_t)(j / ns - 1) & 1u, d.wlim));
        if (!ok) break;
      }
      if (lane == 0) {
        const long long q = chunk_of(j);
        const int c = (int)(q % d.C);
        const long long bh = q / d.C;
        const int h = (int)(bh % d.H), b = (int)(bh / d.H);
        unsigned char* tile = stages + (size_t)(j % ns) * stage_bytes;
        uint64_t* bar = &bar_load[j % ns];
        mbar_expect_tx(bar, (uint32_t)r * (uint32_t)CS * 2u + g.wbytes);
        for (int k = 0; k < r / 8; ++k) tma_load_4d(tile + (size_t)k * g.grp, &mzq, bar, 8 * k, h, c * CS, b);
        bulk_load(tile + g.o_w, wm + (size_t)q * g.wbytes, g.wbytes, bar);
      }
      __syncwarp();
      nload = j + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every copy has landed before the CTA leaves (bounded)
      for (int s = 0; s < ns; ++s) {
        int last = -1;
        for (int j = s; j < nload; j += ns) last = j;
        if (last >= 0) mbar_wait(&bar_load[s], (uint32_t)(last / ns) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- products ----
    const uint32_t id = idesc_bf16(g.mrows, P, false, false);
    const uint32_t lbo_b = (uint32_t)P * 16u;
    int nmma = 0;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_load[j % ns], (uint32_t)(j / ns) & 1u, d.wlim));
      if (ok && j >= kReadBufs)
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_read[j % kReadBufs], (uint32_t)(j / kReadBufs - 1) & 1u, d.wlim));
      if (!ok) break;
      if (lane == 0) {
        fence_after_sync();
        const uint32_t a0 = smem_u32(stages + (size_t)(j % ns) * stage_bytes);
        const uint32_t b0 = a0 + g.o_w;
        const uint32_t acc = tbase + (uint32_t)(j % kReadBufs) * g.ncols;
        for (int part = 0; part < 2; ++part)
          for (int ks = 0; ks < r / 16; ++ks)
            mma_bf16(acc, sdesc(a0 + 2u * g.grp * ks, g.grp, 128u),
                     sdesc(b0 + (uint32_t)part * (uint32_t)(P * r * 2) + 2u * lbo_b * ks, lbo_b, 128u), id,
                     part > 0 || ks > 0);
        mma_commit(&bar_mma[j % kReadBufs]);
      }
      __syncwarp();
      nmma = j + 1;
    }
    if (!ok && lane == 0) atomicExch(&err, 1);
    if (lane == 0) {   // every product has completed before the CTA leaves (bounded)
      for (int s = 0; s < kReadBufs; ++s) {
        int last = -1;
        for (int j = s; j < nmma; j += kReadBufs) last = j;
        if (last >= 0) mbar_wait(&bar_mma[s], (uint32_t)(last / kReadBufs) & 1u, kWaitLimit);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue ----
    const int qd = warp & 3;
    const int m = g.mrows == 64 ? 16 * qd + lane : 32 * qd + lane;
    const bool lane_ok = g.mrows == 128 || lane < 16;
    for (int j = 0; j < nj; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_mma[j % kReadBufs], (uint32_t)(j / kReadBufs) & 1u, d.wlim))) {
        if (lane == 0) atomicExch(&err, 1);
        break;
      }
      fence_after_sync();
      if (warp == 2 && lane == 0) mbar_arrive(&bar_free[j % ns]);   // the products have read the stage
      const long long q = chunk_of(j);
      const int c = (int)(q % d.C);
      const long long bh = q / d.C;
      const int h = (int)(bh % d.H), b = (int)(bh / d.H);
      const int t = c * CS + m;
      const bool live = lane_ok && m < CS && t < T;
      const uint32_t ta = tbase + (uint32_t)(j % kReadBufs) * g.ncols + ((uint32_t)(32 * qd) << 16);
      for (int j0 = 0; j0 < P; j0 += 16) {
        float x[16];
        tmem_ld16(ta + (uint32_t)j0, x);
        if (live) store_y16(y, b, t, h, j0, x, y32);
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_read[j % kReadBufs]);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (err) {   // poison this CTA's chunks
    const float nan = __int_as_float(0x7fc00000);
    float xn[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) xn[e] = nan;
    for (int j = 0; j < nj; ++j) {
      const long long q = chunk_of(j);
      const int c = (int)(q % d.C);
      const long long bh = q / d.C;
      const int h = (int)(bh % d.H), b = (int)(bh / d.H);
      for (int m = tid; m < CS; m += kReadPsThreads) {
        const int t = c * CS + m;
        if (t < T)
          for (int j0 = 0; j0 < P; j0 += 16) store_y16(y, b, t, h, j0, xn, y32);
      }
      if (tid == 0) status[q] |= 1 << 2;
    }
  }
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, kReadBufs * g.ncols);
  }
}

// the readout's conditions on the sizes and on zq (TMA-readable), without y
bool readout_tc_zq_ok(const Dims& d, const In& zq) {
  if (d.r % 16 != 0 || d.r > 64 || d.P % 16 != 0 || d.P > 128 || d.CS % 16 != 0 || d.CS > 128) return false;
  if ((reinterpret_cast<uintptr_t>(zq.p) & 15u) != 0) return false;
  if (!stride_ok(zq.st, d.T) || !stride_ok(zq.sh, d.H) || !stride_ok(zq.sb, d.B)) return false;
  return read_geom(d.r, d.P, d.CS).smem <= 227u * 1024u - 64u;
}

bool readout_tc_ok(const Dims& d, const In& zq, const Out& y) {
  if (!readout_tc_zq_ok(d, zq) || (reinterpret_cast<uintptr_t>(y.p) & 15u) != 0) return false;
  const auto s8 = [](long long s, long long extent) { return extent == 1 || s % 8 == 0; };
  return s8(y.st, d.T) && s8(y.sh, d.H) && s8(y.sb, d.B);
}

cudaError_t launch_readout_tc(const Dims& d, const In& zq, const unsigned char* wm, const Out& y, bool y32,
                              int* status, cudaStream_t st) {
  CUtensorMap mq;
  const ReadGeom g = read_geom(d.r, d.P, d.CS);
  if (!token_map(&mq, zq, d.B, d.T, d.H, d.r, d.CS)) return cudaErrorInvalidValue;
  // persistent CTAs, two per SM, when at least two stages fit in half an SM's shared memory
  // and the TMEM buffers of two CTAs fit the SM's 512 columns
  const uint32_t stage = up128(g.o_w + g.wbytes);
  const int ns = (int)std::min<size_t>(kReadStagesMax, (100u * 1024u - 128u) / stage);
  if (ns >= 2 && 2u * kReadBufs * g.ncols <= kTmemCols) {
    // no third CTA on an SM: its TMEM allocation would wait for a whole other CTA
    const size_t smem = tmem_safe_smem(kReadBufs * g.ncols, kReadPsThreads, (size_t)ns * stage + 128);
    cudaError_t e = cudaFuncSetAttribute(k_readout_ps, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const long long n = (long long)d.B * d.H * d.C;
    const unsigned grid = (unsigned)std::min<long long>(n, 2LL * sms);
    k_readout_ps<<<grid, kReadPsThreads, smem, st>>>(mq, d, g, stage, ns, wm, y, y32, status);
    return cudaGetLastError();
  }
  const size_t smem = tmem_safe_smem(g.ncols, kReadThreads, g.smem);
  cudaError_t e = cudaFuncSetAttribute(k_readout_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H * d.C;
  k_readout_tc<<<(unsigned)n, kReadThreads, smem, st>>>(mq, d, g, wm, y, y32, status);
  return cudaGetLastError();
}

bool stats_scan_tc_ok(const Dims& d, const In& z, const In& v) {
  // r = 32 and 2r + P <= 128: one 128-row product, one 32-float record row per thread
  return (long long)d.B * d.H >= 64 && d.r == 32 && 2 * d.r + d.P <= 128 && stats_tc_ok(d, z, v);
}

cudaError_t launch_stats_scan_tc(const Dims& d, const In& z, const In& v, float* stats, unsigned long long* cmax,
                                 int* status, cudaStream_t st) {
  CUtensorMap mz, mv;
  StatsGeom g = stats_geom(d.r, d.P, d.CS);
  if (!token_map(&mz, z, d.B, d.T, d.H, d.r, d.CS, g.sw) || !token_map(&mv, v, d.B, d.T, d.H, d.P, d.CS, g.sw))
    return cudaErrorInvalidValue;
  // as many copy stages as fit next to the record warps' tiles (2 .. kScanStagesMax)
  const size_t tile_bytes = (size_t)g.nb * (g.sw ? 4 : 16) * g.grp, fixed = 4 * 4096 + 1024;
  const int ns = (int)std::min<size_t>(kScanStagesMax, (200u * 1024u - fixed) / tile_bytes);
  if (ns < 2) return cudaErrorInvalidValue;
  g.smem = (size_t)ns * tile_bytes + fixed;
  uint32_t c = 32;
  while (c < (uint32_t)(kScanBufs * g.nb * d.r)) c <<= 1;   // the product buffers
  g.ncols = c;
  cudaError_t e = cudaFuncSetAttribute(k_stats_scan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return e;
  k_stats_scan_tc<<<(unsigned)((long long)d.B * d.H), kScanThreads, g.smem, st>>>(mz, mv, d, g, ns, stats, cmax,
                                                                                 status);
  return cudaGetLastError();
}

cudaError_t launch_stats_tc(const Dims& d, const In& z, const In& v, float* stats, unsigned long long* cmax,
                            int* status, cudaStream_t st) {
  CUtensorMap mz, mv;
  const StatsGeom g = stats_geom(d.r, d.P, d.CS);
  if (!token_map(&mz, z, d.B, d.T, d.H, d.r, d.CS, g.sw) || !token_map(&mv, v, d.B, d.T, d.H, d.P, d.CS, g.sw))
    return cudaErrorInvalidValue;
  const size_t smem = tmem_safe_smem(g.ncols, kStatsThreads, g.smem);
  cudaError_t e = cudaFuncSetAttribute(k_stats_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H * d.C;
  k_stats_tc<<<(unsigned)n, kStatsThreads, smem, st>>>(mz, mv, d, g, stats, cmax, status);
  return cudaGetLastError();
}

}  // namespace tc
}  // namespace ska
