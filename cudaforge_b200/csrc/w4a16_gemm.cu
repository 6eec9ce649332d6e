// W4A16 group-128 GEMM (and the dense bf16/fp16 variant) on sm_100a tensor
// cores: tcgen05.mma with the accumulator in TMEM, TMA-staged operands.
//
// Replaces the reference's INT4 GEMM interface
// (csrc/include/cudaforge/kernels/dequantize.cuh:12-31,
//  csrc/kernels/cuda/int4_gemm_dequant.cu:37-133,
//  csrc/kernels/triton/int4_dequant_triton.py:7-131):
//     Y[M, N] = X[M, K] . deq(Wq)[K, N],  deq = (nibble - 8) * scale[k / 128, n]
// with Wq the reference's [K/8, N] uint32 packing (nibble i of word (j, n)
// holds k = 8j + i, tests/unit/test_int4_dequant.py:6-15) and zero point 8
// (signed INT4, the `zeros == 8` case of int4_gemm_dequant.cu:87-92).
//
// Design (swap-AB, because M = tokens is small and N*K = weights is large):
//   the MMA computes D^T[n, m] = W[n, :] . X[m, :]; weight rows are the
//   tcgen05 "A" operand (M = 128 per MMA) and the token tile (<= 256 tokens
//   x 64 k) the "B" operand.  One CTA = 256 weight rows (two 128-row MMA
//   halves, two TMEM accumulators) x one K split x one token slice, so each
//   token tile the SM pulls through its TMA path feeds 256 weight rows: the
//   per-SM TMA path (~100 GB/s from L2, ~0.1-0.3 us per op from one issuing
//   thread, measured) is what the tile shape is sized against.  19 warps:
//     warp 0      weight producer (lane 0 packed W, lane 1 group scales)
//     warp 1      TMEM allocator + MMA issue (one thread)
//     warps 2-17  INT4 -> bf16 dequantisation straight into TMEM (one weight
//                 row per thread; two groups of 8 warps take alternate
//                 stages), then the epilogue
//                 (tcgen05.ld -> shared staging -> 16-byte row-contiguous
//                 stores)
//     warp 18     token-tile producer
//   Three independent rings (packed W, dequantised A, token tile), every
//   mbarrier wait bounded (a device status word records CF_ETIMEOUT), no TMA
//   multicast.
//
// The packed weights are consumed in a kernel-native nibble order produced
// once per weight by cf_w4a16_repack (the same values; see dequant8()).
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

#include <algorithm>
#include <mutex>
#include <cstdlib>

namespace {

using namespace cf::sm100;

constexpr int kDqGroups = 2;                    // dequantisation warp groups (8 warps each, alternate stages)
constexpr int kXWarp = 2 + 8 * kDqGroups;       // token-tile producer warp
constexpr int kThreads = (kXWarp + 1) * 32;     // 19 warps
constexpr int HN = 128;        // weight rows per MMA (tcgen05 M)
constexpr int TN = 256;        // weight rows per CTA (two MMA halves)
constexpr int BK = 64;         // k per pipeline stage: one 128-B swizzle atom of 16-bit elements
constexpr int kMaxSlice = 256; // tokens per CTA (MMA N), two accumulators fit 512 TMEM columns
constexpr int kMaxSmem = 232448;
constexpr uint32_t kHalfBytes = HN * BK * 2;           // 16 KB dequantised half tile
constexpr uint32_t kAStageBytes = 2 * kHalfBytes;      // 32 KB
constexpr uint32_t kWPackBytes = (BK / 8) * TN * 4;    // 8 KB packed INT4
constexpr uint32_t kScaleBytes = TN * 2;               // 512 B fp16 group scales
constexpr uint32_t kWStageBytes = kWPackBytes + kScaleBytes;
constexpr uint64_t kDrainNs = 1000000000ull;

enum WMode : int { kInt4 = 0, kDense = 1 };

struct GemmParams {
  int M, N, K;
  int m_slice, kb_per_split, splits;
  int sa, sx, sw;                  // ring depths: dequantised A, token tile X, packed W (+scales)
  uint32_t off_x, off_w, off_bar;  // ring bases (A ring at 0)
  uint32_t x_bytes;
  int x_box;                       // token rows per TMA box (divides m_slice)
  uint32_t tmem_cols, idesc;
  uint32_t a_tcol;                 // INT4: first TMEM column of the dequantised-A stages
  void *y;
  int64_t ldy;
  const void *residual;
  int64_t ldr;
  float *partial;
  int *status;
  uint64_t timeout_ns;
  unsigned long long *trace;
};

// 8 repacked nibbles -> 8 bf16 (k order 0..7).  Repacked nibble position p
// holds k = 2p for p < 4 and k = 2(p-4)+1 for p >= 4, so masking with
// 0x000F000F after shifts of 0/4/8/12 yields the pairs (k0,k1) (k2,k3)
// (k4,k5) (k6,k7).  OR-ing 0x4300 builds bf16 128 + nibble exactly;
// subtracting 136 gives v = nibble - 8 exactly.
// The weight is bf16(v * s) with ONE rounding of the exact product, as the
// reference dequantises in fp32 and then casts to the activation type
// (csrc/kernels/triton/int4_dequant_triton.py:66).  The fp16 scale s (11
// significant bits) is split as s = s_hi + s_lo with s_hi = bf16(s) and s_lo
// = s - s_hi (at most 3 significant bits, exact in bf16); v * s_lo has at most
// 6 significant bits and is exact in bf16, so fma(v, s_hi, v * s_lo) rounds
// v * s exactly once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __nv_bfloat162 s_hi, __nv_bfloat162 s_lo) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u;
  const __nv_bfloat162 k136 = __floats2bfloat162_rn(136.0f, 136.0f);
  uint32_t h[4] = {(w & kMask) | kMagic, ((w >> 4) & kMask) | kMagic, ((w >> 8) & kMask) | kMagic,
                   ((w >> 12) & kMask) | kMagic};
  uint4 o;
  uint32_t *op = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&h[j]);
    v = __hsub2(v, k136);
    v = __hfma2(v, s_hi, __hmul2_rn(v, s_lo));
    op[j] = *reinterpret_cast<uint32_t *>(&v);
  }
  return o;
}

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Optional per-role timeline of CTA (0,0,0) (cf_gemm_args.trace).
#define CF_TRACE(role, i) \
  if (tr && (i) < 512) p.trace[(role) * 512 + (i)] = clock64()

// MMA issue of one CTA (one thread): per 64-k stage, 4 k-steps x H weight-row halves.
template <int WM, int H>
__device__ __forceinline__ bool mma_loop(const GemmParams &p, uint32_t tmem, uint8_t *a_ring, uint8_t *x_ring,
                                         uint64_t *afull, uint64_t *xfull, uint64_t *aempty, uint64_t *xempty,
                                         int nkb, bool tr) {
  // parameters copied to registers once: every inline-asm statement below clobbers
  // memory, which would otherwise force a reload of each field after every MMA
  const uint32_t idesc = p.idesc;
  const int SA = p.sa, SX = p.sx;
  const uint32_t m_slice = (uint32_t)p.m_slice, a_tcol = p.a_tcol, x_bytes = p.x_bytes;
  const uint64_t limit = p.timeout_ns;
  int sa = 0, sx = 0;
  uint32_t pa = 0, px = 0;
  for (int i = 0; i < nkb; ++i) {
    CF_TRACE(6, i);
    if (!mbar_wait(&afull[sa], pa, limit)) return false;
    CF_TRACE(7, i);
    if (!mbar_wait(&xfull[sx], px, limit)) return false;
    tc_fence_after();
    const uint32_t a_base = smem_u32(a_ring + sa * kAStageBytes);
    const uint32_t x_base = smem_u32(x_ring + sx * x_bytes);
    const uint32_t at0 = tmem + a_tcol + (uint32_t)(sa * 64);
    CF_TRACE(3, i);
#pragma unroll
    for (int k16 = 0; k16 < BK / 16; ++k16) {
      const uint64_t bd = desc_kmajor_sw128(x_base + k16 * 32);
      const uint32_t acc = (i > 0 || k16 > 0) ? 1u : 0u;
#pragma unroll
      for (int h = 0; h < H; ++h) {
        if (WM == kInt4)  // A from TMEM: 32 columns per half per stage, 8 per k16
          mma_f16_ts(tmem + (uint32_t)h * m_slice, at0 + (uint32_t)(h * 32 + k16 * 8), bd, idesc, acc);
        else
          mma_f16(tmem + (uint32_t)h * m_slice, desc_kmajor_sw128(a_base + h * kHalfBytes + k16 * 32), bd, idesc,
                  acc);
      }
    }
    // one commit per stage: xempty[] is the ring of stage-done barriers that the token
    // producer and the A-slot writers both wait on (depth SX >= SA)
    mma_commit(&xempty[sx]);
    CF_TRACE(8, i);
    if (++sa == SA) { sa = 0; pa ^= 1u; }
    if (++sx == SX) { sx = 0; px ^= 1u; }
  }
  return true;
}

template <typename T, int WM>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
            const __grid_constant__ CUtensorMap tm_s, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SA = p.sa, SX = p.sx, SW = p.sw;
  uint8_t *a_ring = smem;                 // SA x 32 KB weight tiles (two 128-row halves)
  uint8_t *x_ring = smem + p.off_x;       // SX x x_bytes token tiles
  uint8_t *w_ring = smem + p.off_w;       // SW x (8 KB packed + 512 B scales), INT4 only
  uint64_t *wfull = reinterpret_cast<uint64_t *>(smem + p.off_bar);
  uint64_t *wempty = wfull + SW;
  uint64_t *xfull = wempty + SW;
  uint64_t *xempty = xfull + SX;
  uint64_t *afull = xempty + SX;
  uint64_t *aempty = afull + SA;
  uint64_t *accf = aempty + SA;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * p.m_slice;
  const int n0 = blockIdx.y * TN;
  const int split = blockIdx.z;
  const int halves = (n0 + HN < p.N) ? 2 : 1;
  const int mrows = min(p.m_slice, p.M - m0);
  const int kbs = p.K / BK;
  const int kb0 = split * p.kb_per_split;
  const int nkb = min(p.kb_per_split, kbs - kb0);
  // Rotated k order: CTAs start at different k-blocks so they do not all read the
  // same token-tile lines of L2 at the same moment (each CTA's order is fixed).
  const int rot = nkb > 0 ? (int)((blockIdx.y * 7u + blockIdx.x * 3u) % (unsigned)nkb) : 0;
  auto kb_of = [&](int i) { int j = i + rot; return kb0 + (j >= nkb ? j - nkb : j); };
  const bool tr = p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  if (threadIdx.x == 0) CF_TRACE(5, 2);  // kernel entry

  // set when any role's bounded wait ran out: every role then drains before TMEM is freed
  volatile int &s_fail = *reinterpret_cast<volatile int *>(tmem_slot + 1);
  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < SW; ++s) { mbar_init(&wfull[s], 1); mbar_init(&wempty[s], 8); }
    for (int s = 0; s < SX; ++s) { mbar_init(&xfull[s], 1); mbar_init(&xempty[s], 1); }
    for (int s = 0; s < SA; ++s) { mbar_init(&afull[s], WM == kInt4 ? 8 : 1); mbar_init(&aempty[s], 1); }
    mbar_init(accf, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    if (WM == kInt4) prefetch_tmap(&tm_s);
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued_w = 0, issued_x = 0;  // copies this CTA's producers started (drained on failure)

  if (warp == 0) {
    // ---------------- weight producer ----------------
    const int S = WM == kInt4 ? SW : SA;
    uint64_t *fullb = WM == kInt4 ? wfull : afull;
    uint64_t *emptyb = WM == kInt4 ? wempty : aempty;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (WM == kInt4) {
        if (i >= S && !mbar_wait_warp(&emptyb[s], ph ^ 1u, p.timeout_ns)) { ok = false; break; }
      } else if (i >= SA) {  // dense: A slot s is free once stage i - SA is done
        const int j = i - SA;
        if (!mbar_wait_warp(&xempty[j % SX], (uint32_t)(j / SX) & 1u, p.timeout_ns)) { ok = false; break; }
      }
      const int kb = kb_of(i);
      if (lane == 0) {
        CF_TRACE(0, i);
        mbar_arrive_expect_tx(&fullb[s], WM == kInt4 ? kWStageBytes : (uint32_t)halves * kHalfBytes);
      }
      __syncwarp();
      // The issuing lane rotates with the stage: one thread's TMA copies were measured
      // not to overlap one another, copies from different threads do.
      const int l0 = (2 * i) & 31;
      if (WM == kInt4) {
        uint8_t *st = w_ring + s * kWStageBytes;
        if (lane == l0) tma_load_2d(st, &tm_w, &fullb[s], n0, kb * (BK / 8));
        if (lane == l0 + 1) tma_load_2d(st + kWPackBytes, &tm_s, &fullb[s], n0, (kb * BK) / 128);
      } else {
        if (lane >= l0 && lane < l0 + halves)
          tma_load_2d(a_ring + s * kAStageBytes + (lane - l0) * kHalfBytes, &tm_w, &fullb[s], kb * BK,
                      n0 + (lane - l0) * HN);
      }
      __syncwarp();
      issued_w = i + 1;
    }
  } else if (warp == kXWarp) {
    // ---------------- token-tile producer ----------------
    for (int i = 0; i < nkb; ++i) {
      const int s = i % SX;
      const uint32_t ph = (uint32_t)(i / SX) & 1u;
      if (i >= SX && !mbar_wait_warp(&xempty[s], ph ^ 1u, p.timeout_ns)) { ok = false; break; }
      const int kb = kb_of(i);
      // boxes of x_box token rows (x_box * 128 B, 1024-B aligned; the 128-B swizzle
      // pattern repeats every 8 rows, so any multiple of 8 rows gives the layout of one
      // tile), one per lane, rotating over the lanes per stage.  The per-SM TMA unit is
      // bound by operations more than bytes: few large boxes feed it fastest.
      if (lane == 0) {
        CF_TRACE(4, i);
        mbar_arrive_expect_tx(&xfull[s], p.x_bytes);
      }
      __syncwarp();
      {
        const int nbox = p.m_slice / p.x_box;
        const int b = (lane - i * nbox) & 31;  // box handled by this lane (rotating per stage)
        if (b < nbox)
          tma_load_2d(x_ring + s * p.x_bytes + b * p.x_box * 128, &tm_x, &xfull[s], kb * BK, m0 + b * p.x_box);
      }
      __syncwarp();
      issued_x = i + 1;
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: one thread; ring slots and phases advance by increments ----------------
    // The stage's MMAs are a compile-time unrolled block (the number of halves is a
    // template argument): measured on B200, a runtime-bounded loop around tcgen05.mma
    // and tcgen05.commit ran at 250-450 cycles per MMA, the unrolled block at the
    // tensor pipe's rate (~96 cycles at M=128, N=192, K=16).
    if (lane == 0) {
      if (halves == 2) ok = mma_loop<WM, 2>(p, tmem, a_ring, x_ring, afull, xfull, aempty, xempty, nkb, tr);
      else ok = mma_loop<WM, 1>(p, tmem, a_ring, x_ring, afull, xfull, aempty, xempty, nkb, tr);
      mma_commit(accf);  // completes when every issued MMA has finished
    }
    __syncwarp();
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  } else {
    // ---------------- dequantisation (warps 2-17) straight into TMEM ----------------
    // Warp w may only touch TMEM lanes 32*(w%4)..+31, so warp w owns rows
    // (w%4)*32 + lane of half h = ((w-2)/4)%2; each thread dequantises its row's
    // 64 k values and stores them with one tcgen05.st (32 columns).  Group
    // g = (w-2)/8 takes the stages i = g (mod 2): one group's dequantisation of a stage
    // (~850 cycles, latency-bound at two warps per SM sub-partition) overlaps the other's.
    const int q = warp & 3, h = ((warp - 2) >> 2) & 1, g = (warp - 2) >> 3;
    const int row = q * 32 + lane;  // within the half == TMEM lane
    const int t = h * HN + row;     // within the 256-row tile
    if (WM == kInt4) {
      for (int i = g; i < nkb; i += kDqGroups) {
        const int sw = i % SW;
        // warp-uniform waits: a lane must not leave the loop while the others reach __syncwarp
        if (!mbar_wait_warp(&wfull[sw], (uint32_t)(i / SW) & 1u, p.timeout_ns)) { ok = false; break; }
        if (threadIdx.x == 64) CF_TRACE(9, i);
        const uint8_t *st = w_ring + sw * kWStageBytes;
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(st);
        const float sf = __half2float(reinterpret_cast<const __half *>(st + kWPackBytes)[t]);
        const __nv_bfloat16 sh = __float2bfloat16_rn(sf);
        const __nv_bfloat16 sl = __float2bfloat16_rn(sf - __bfloat162float(sh));  // exact remainder
        const __nv_bfloat162 s_hi = __halves2bfloat162(sh, sh), s_lo = __halves2bfloat162(sl, sl);
        uint32_t a[32];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint4 v = dequant8(wp[kk * TN + t], s_hi, s_lo);
          a[4 * kk + 0] = v.x; a[4 * kk + 1] = v.y; a[4 * kk + 2] = v.z; a[4 * kk + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[sw]);  // packed words are consumed
        // dequantised into registers first: only the TMEM store waits for the A slot
        const int sa = i % SA;
        if (threadIdx.x == 64) CF_TRACE(10, i);
        // A slot sa is free once stage i - SA is done (the stage-done ring has depth SX >= SA)
        if (i >= SA && !mbar_wait_warp(&xempty[(i - SA) % SX], (uint32_t)((i - SA) / SX) & 1u, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == 64) CF_TRACE(1, i);
        if (h < halves)
          tmem_st_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + p.a_tcol + (uint32_t)((sa * 2 + h) * 32), a);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[sa]);
        if (threadIdx.x == 64) CF_TRACE(2, i);
      }
    }
    // ---------------- epilogue ----------------
    if (!mbar_wait_warp(accf, 0, ok ? p.timeout_ns : kDrainNs)) ok = false;
    tc_fence_after();
    if (threadIdx.x == 64) CF_TRACE(5, 0);
    if (ok) {
      // TMEM row (this lane) x 32 token columns -> a per-warp staging tile in the (now idle)
      // A ring, then 16-byte row-contiguous stores: each token row's 32 outputs are 64 B
      // (bf16) or 128 B (fp32 partials) of one global row.
      float *stg = reinterpret_cast<float *>(a_ring + (warp - 2) * 4096);  // [32 tokens][32 n]
      T *y = reinterpret_cast<T *>(p.y);
      const T *res = reinterpret_cast<const T *>(p.residual);
      if (h < halves) {  // per group: 4 warps drain half 0, 4 half 1; the groups alternate 32-token chunks
        const int nw = n0 + h * HN + q * 32;
        for (int c = 32 * g; c < mrows; c += 32 * kDqGroups) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * p.m_slice + c), r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = __uint_as_float(r[j]);
          __syncwarp();
          const int lim = min(32, mrows - c);
#pragma unroll
          for (int pass = 0; pass < 8; ++pass) {
            const int j = pass * 4 + (lane >> 3);  // token within the 32
            const int nn = (lane & 7) * 4;         // 4 consecutive outputs
            if (j < lim) {
              const float4 v = *reinterpret_cast<const float4 *>(stg + j * 32 + nn);
              const int64_t m = m0 + c + j;
              if (p.splits > 1) {
                *reinterpret_cast<float4 *>(p.partial + ((int64_t)split * p.M + m) * p.N + nw + nn) = v;
              } else {
                float o[4] = {v.x, v.y, v.z, v.w};
                if (res) {
                  const uint2 rr = *reinterpret_cast<const uint2 *>(res + m * p.ldr + nw + nn);
                  const T *rp = reinterpret_cast<const T *>(&rr);
#pragma unroll
                  for (int e = 0; e < 4; ++e) o[e] += cf::to_float(rp[e]);
                }
                uint2 w;
                T *wp = reinterpret_cast<T *>(&w);
#pragma unroll
                for (int e = 0; e < 4; ++e) wp[e] = from_f<T>(o[e]);
                *reinterpret_cast<uint2 *>(y + m * p.ldy + nw + nn) = w;
              }
            }
          }
          __syncwarp();
        }
      }
    }
  }
  if (!ok) s_fail = 1;
  __syncthreads();
  if (s_fail) {
    // Some wait ran out, so other roles may have stopped early: before the CTA can
    // exit, let this CTA's own TMA copies land and every MMA it issued finish
    // (all bounded), then free TMEM.
    if (warp == 0) {
      const int S = WM == kInt4 ? SW : SA;
      uint64_t *fullb = WM == kInt4 ? wfull : afull;
      for (int j = max(0, issued_w - S); j < issued_w; ++j)
        mbar_wait_warp(&fullb[j % S], (uint32_t)(j / S) & 1u, kDrainNs);
    } else if (warp == kXWarp) {
      for (int j = max(0, issued_x - SX); j < issued_x; ++j)
        mbar_wait_warp(&xfull[j % SX], (uint32_t)(j / SX) & 1u, kDrainNs);
    } else if (warp == 1) {
      mbar_wait_warp(accf, 0, kDrainNs);
    }
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, CF_ETIMEOUT);
  }
  if (threadIdx.x == 64) CF_TRACE(5, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// Fixed-order split-K reduction with the optional residual fused:
//   y[m, n] = sum_{s < splits} partial[s, m, n] (+ residual[m, n])
template <typename T>
__global__ void splitk_reduce_kernel(const float *partial, int splits, int M, int N, T *y, int64_t ldy,
                                     const T *res, int64_t ldr) {
  const int64_t total4 = (int64_t)M * N / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    const int64_t m = e / N, n = e % N;
    float4 acc = reinterpret_cast<const float4 *>(partial)[i];
    for (int s = 1; s < splits; ++s) {
      const float4 v = reinterpret_cast<const float4 *>(partial + (int64_t)s * M * N)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (res) {
      const T *r = res + m * ldr + n;
      acc.x += cf::to_float(r[0]); acc.y += cf::to_float(r[1]);
      acc.z += cf::to_float(r[2]); acc.w += cf::to_float(r[3]);
    }
    T *d = y + m * ldy + n;
    d[0] = from_f<T>(acc.x); d[1] = from_f<T>(acc.y); d[2] = from_f<T>(acc.z); d[3] = from_f<T>(acc.w);
  }
}

// Reference packing -> kernel nibble order (see dequant8).
__global__ void repack_kernel(const uint32_t *src, uint32_t *dst, int64_t n_words) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_words; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t w = src[i];
    uint32_t o = 0;
#pragma unroll
    for (int pos = 0; pos < 8; ++pos) {
      const int k = pos < 4 ? 2 * pos : 2 * (pos - 4) + 1;
      o |= ((w >> (4 * k)) & 0xFu) << (4 * pos);
    }
    dst[i] = o;
  }
}

struct Plan {
  int slices, m_slice, splits, kb_per_split, sa, sx, sw, ntiles, x_box;
  uint32_t x_bytes, off_x, off_w, off_bar, tmem_cols, a_tcol;
  size_t smem;
};

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  return sms;
}

bool make_plan(int M, int N, int K, int split_req, bool int4, Plan &pl) {
  // INT4: TMEM = two accumulators (2 x m_slice columns) + >= 2 dequantised-A stages (64 columns each)
  const int max_slice = int4 ? 192 : kMaxSlice;
  pl.slices = (M + max_slice - 1) / max_slice;
  const int per = (M + pl.slices - 1) / pl.slices;
  pl.m_slice = (per + 15) / 16 * 16;
  if (pl.m_slice > max_slice) return false;
  pl.x_box = pl.m_slice;  // one TMA box per token tile (box rows <= 256)
  // smem: A ring (dense: 32 KB / stage; INT4: 64 KB epilogue staging) | X ring | W ring (8.5 KB / stage)
  pl.x_bytes = (uint32_t)pl.m_slice * 128u;
  const size_t budget = kMaxSmem - 1024 - 1024;  // alignment slack + barriers
  const size_t w_stage = int4 ? kWStageBytes : 0;
  if (int4) {
    pl.a_tcol = (2u * pl.m_slice + 31u) & ~31u;
    pl.sa = std::min(4, (int)((512u - pl.a_tcol) / 64u));
    pl.tmem_cols = 512;
  } else {
    pl.a_tcol = 0;
    pl.sa = 3;
  }
  // INT4: the A ring's smem is only the epilogue staging, 4 KB per dequantisation warp
  const size_t stage_bytes = (size_t)kDqGroups * 8 * 4096;
  const size_t a_bytes = int4 ? stage_bytes : pl.sa * (size_t)kAStageBytes;
  pl.sw = int4 ? 8 : 1;
  pl.sx = (int)std::min<size_t>(6, (budget - a_bytes - pl.sw * w_stage) / pl.x_bytes);
  if (pl.sx < 2 && !int4) { pl.sa = 2; pl.sx = (int)std::min<size_t>(4, (budget - 2 * (size_t)kAStageBytes) / pl.x_bytes); }
  if (pl.sx < 2 || pl.sa < 2 || (int4 && pl.sw < 2)) return false;
  pl.sa = std::min(pl.sa, pl.sx);  // stage-done barriers live in the X ring (depth SX >= SA)
  pl.off_x = (uint32_t)a_bytes;
  pl.off_w = pl.off_x + pl.sx * pl.x_bytes;
  pl.off_bar = (pl.off_w + (int4 ? pl.sw * kWStageBytes : 0) + 15u) & ~15u;
  pl.smem = 1024 + pl.off_bar + 8 * (2 * pl.sw + 2 * pl.sx + 2 * pl.sa + 1) + 16;
  if (!int4) {
    uint32_t cols = 32;
    while (cols < 2u * (uint32_t)pl.m_slice) cols <<= 1;
    pl.tmem_cols = cols;
  }
  const int kbs = K / BK;
  pl.ntiles = (N + TN - 1) / TN;
  const int tiles = pl.ntiles * pl.slices;
  int splits = split_req > 0 ? split_req : std::max(1, num_sms() / tiles);
  splits = std::max(1, std::min(splits, kbs / 2 > 0 ? kbs / 2 : 1));
  pl.kb_per_split = (kbs + splits - 1) / splits;
  pl.splits = (kbs + pl.kb_per_split - 1) / pl.kb_per_split;
  return true;
}

// partials_only: when the plan splits K, leave the fp32 partials [splits][m][n] in the
// workspace for a fused consumer (cf_splitk_*) instead of launching the reduction.
template <typename T, int WM>
int run_gemm(const cf_gemm_args &a, cudaStream_t stream, bool partials_only = false) {
  const bool int4 = WM == kInt4;
  if (a.m < 0 || a.n <= 0 || a.k <= 0) return CF_EINVAL;
  if (a.m == 0) return CF_OK;
  if (a.n % HN != 0 || a.k % (int4 ? 128 : BK) != 0) return CF_EINVAL;
  if (!a.x || !a.w || !a.y || (int4 && !a.scales)) return CF_EINVAL;
  if (a.ldx < a.k || a.ldy < a.n || (a.residual && a.ldr < a.n)) return CF_EINVAL;
  // the epilogue writes 4 outputs (8 B) per vector store
  if (a.ldy % 4 || (a.residual && a.ldr % 4) || (reinterpret_cast<uintptr_t>(a.y) & 7) ||
      (reinterpret_cast<uintptr_t>(a.residual) & 7))
    return CF_EINVAL;
  Plan pl;
  if (!make_plan(a.m, a.n, a.k, a.split_k, int4, pl)) return CF_EUNSUPPORTED;
  if (pl.splits > 1) {
    const size_t need = (size_t)pl.splits * a.m * a.n * sizeof(float);
    if (!a.workspace || a.workspace_bytes < need) return CF_EINVAL;
    if ((reinterpret_cast<uintptr_t>(a.workspace) & 15) != 0 || a.n % 4 != 0) return CF_EINVAL;
    if (a.residual && (a.ldr % 4) != 0) return CF_EINVAL;
  }
  const CUtensorMapDataType tdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tx, tw, ts;
  if (!cf::make_tmap_2d(&tx, tdt, a.x, (uint64_t)a.k, (uint64_t)a.m, (uint64_t)a.ldx * 2, BK, (uint32_t)pl.x_box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
    return CF_EINVAL;
  if (int4) {
    if (!cf::make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, (uint64_t)a.n, (uint64_t)a.k / 8,
                          (uint64_t)a.n * 4, TN, BK / 8, CU_TENSOR_MAP_SWIZZLE_NONE))
      return CF_EINVAL;
    if (!cf::make_tmap_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.scales, (uint64_t)a.n, (uint64_t)a.k / 128,
                          (uint64_t)a.n * 2, TN, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return CF_EINVAL;
  } else {
    if (!cf::make_tmap_2d(&tw, tdt, a.w, (uint64_t)a.k, (uint64_t)a.n, (uint64_t)a.k * 2, BK, HN,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return CF_EINVAL;
    ts = tw;
  }
  GemmParams p;
  p.M = a.m; p.N = a.n; p.K = a.k;
  p.m_slice = pl.m_slice;
  p.kb_per_split = pl.kb_per_split; p.splits = pl.splits;
  p.sa = pl.sa; p.sx = pl.sx; p.sw = pl.sw;
  p.x_box = pl.x_box;
  p.off_x = pl.off_x; p.off_w = pl.off_w; p.off_bar = pl.off_bar; p.x_bytes = pl.x_bytes;
  p.tmem_cols = pl.tmem_cols;
  p.a_tcol = pl.a_tcol;
  p.idesc = cf::sm100::idesc_bf16_f32(HN, pl.m_slice);
  if (std::is_same<T, __half>::value) p.idesc &= ~((7u << 7) | (7u << 10));  // A, B format f16
  p.y = a.y; p.ldy = a.ldy; p.residual = a.residual; p.ldr = a.ldr;
  p.partial = reinterpret_cast<float *>(a.workspace);
  p.status = a.status;
  p.timeout_ns = a.timeout_ns ? a.timeout_ns : 2000000000ull;
  p.trace = reinterpret_cast<unsigned long long *>(a.trace);
  auto kern = gemm_kernel<T, WM>;
  // The dynamic shared memory of a launch depends on the plan (token slice), but the
  // function attribute is per kernel function: raise it once per device to the largest
  // plan and never lower it, or a CUDA graph captured with a larger plan would fail to
  // replay after a smaller plan's launch had lowered the limit.
  {
    static std::mutex mu;
    static bool raised[64][2][2];
    int dev = 0;
    CF_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    bool &done = raised[dev & 63][std::is_same<T, __half>::value][WM];
    if (!done) {
      CF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
      done = true;
    }
  }
  if (pl.smem > (size_t)kMaxSmem) return CF_EINVAL;
  dim3 grid(pl.slices, pl.ntiles, pl.splits);
  kern<<<grid, kThreads, pl.smem, stream>>>(tx, tw, ts, p);
  if (cudaGetLastError() != cudaSuccess) return CF_ECUDA;
  if (pl.splits > 1 && !partials_only) {
    const int64_t total4 = (int64_t)a.m * a.n / 4;
    const int blocks = (int)std::min<int64_t>((total4 + 255) / 256, (int64_t)num_sms() * 8);
    splitk_reduce_kernel<T><<<blocks, 256, 0, stream>>>(p.partial, pl.splits, a.m, a.n, reinterpret_cast<T *>(a.y),
                                                        a.ldy, reinterpret_cast<const T *>(a.residual), a.ldr);
  }
  return cf_launch_status();
}

}  // namespace

extern "C" size_t cf_gemm_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t split_k, int32_t int4) {
  Plan pl;
  if (m <= 0 || n <= 0 || k <= 0 || !make_plan(m, n, k, split_k, int4 != 0, pl)) return 0;
  return pl.splits > 1 ? (size_t)pl.splits * m * n * sizeof(float) : 0;
}

extern "C" int cf_w4a16_gemm(const cf_gemm_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  if (args->act_dtype != CF_BF16) return CF_EUNSUPPORTED;
  return run_gemm<__nv_bfloat16, kInt4>(*args, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int cf_dense_gemm(const cf_gemm_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (args->act_dtype == CF_BF16) return run_gemm<__nv_bfloat16, kDense>(*args, s);
  if (args->act_dtype == CF_F16) return run_gemm<__half, kDense>(*args, s);
  return CF_EUNSUPPORTED;
}

extern "C" int cf_gemm_splits(int32_t m, int32_t n, int32_t k, int32_t split_k, int32_t int4) {
  Plan pl;
  if (m <= 0 || n <= 0 || k <= 0 || n % HN != 0 || k % (int4 ? 128 : BK) != 0) return 0;  // as run_gemm
  if (!make_plan(m, n, k, split_k, int4 != 0, pl)) return 0;
  return pl.splits;
}

extern "C" int cf_w4a16_gemm_partials(const cf_gemm_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  if (args->act_dtype != CF_BF16) return CF_EUNSUPPORTED;
  return run_gemm<__nv_bfloat16, kInt4>(*args, reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int cf_dense_gemm_partials(const cf_gemm_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (args->act_dtype == CF_BF16) return run_gemm<__nv_bfloat16, kDense>(*args, s, true);
  if (args->act_dtype == CF_F16) return run_gemm<__half, kDense>(*args, s, true);
  return CF_EUNSUPPORTED;
}

extern "C" int cf_w4a16_repack(const uint32_t *wq_ref, uint32_t *wq_out, int32_t k, int32_t n, void *stream) {
  if (!wq_ref || !wq_out || k <= 0 || n <= 0 || k % 8 != 0) return CF_EINVAL;
  const int64_t words = (int64_t)(k / 8) * n;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 4096);
  repack_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(wq_ref, wq_out, words);
  return cf_launch_status();
}
