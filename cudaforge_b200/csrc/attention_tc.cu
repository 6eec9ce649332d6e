// Paged verify attention on tcgen05 for wide row groups (sm_100a): the
// (new row x head-in-group) rows of one kv head number >= 128, as in the
// 64-node draft trees of 8B tree verification (65 rows x 4 heads = 260 rows
// per kv head).  Same contract and semantics as verify_attn_kernel in
// attention.cu (reference online-softmax attention,
// csrc/kernels/triton/flash_attn_triton.py:7-110, over the paged
// KVCacheBatchDescriptor layout, csrc/include/cudaforge/memory/
// paged_kv_cache.h:81-94, with the tree-ancestor or causal mask over this
// step's new rows); at these row counts the warp-MMA kernel is bound by its
// tensor throughput, so here both products run on the 5th-generation tensor
// cores with their accumulators in TMEM:
//
//   one CTA = 128 query rows (one row tile of one (sequence, kv head)) x the
//   whole key range, in blocks of 128 keys (8 pages of 16, then one block of
//   this step's new rows);
//   S_j = Q K_j^T   tcgen05.mma, A = Q (smem, K-major), B = K block (smem,
//                   K-major), D = S buffer j%2 in TMEM (128 x 128 fp32);
//   softmax         two groups of 4 warps take alternate blocks (two softmax warps
//                   per SM sub-partition hide each other's latency); one query row
//                   per thread (TMEM lane): row max, 2^(s*scale*log2e - m), row
//                   sum, P_j as bf16 written over S_j's first 64 columns; each group
//                   keeps its own running max, sum and O, raising the max lazily
//                   (only when a block's max exceeds it by more than 2^8, rescaling
//                   that group's O in TMEM then);
//   O_g += P_j V_j  tcgen05.mma, A = P_j (TMEM), B = V block (smem, MN-major),
//                   D = O of group g = j % 2 in TMEM (128 x 128 fp32);
//   output          the two groups merged per row in log-sum-exp form, O / l, bf16.
// TMEM: S/P buffer 0 [0,128), 1 [128,256), O of group 0 [256,384), group 1 [384,512).
// Warps: 0 K producer and 10 V producer (TMA page boxes; the new rows as one 3-D box
// each), 1 TMEM allocator + MMA issue (one thread), 2-5 and 6-9 softmax groups.  Every
// mbarrier wait is bounded (CF_ETIMEOUT in the status word); no multicast.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

#include <math.h>

namespace cf {
namespace attn_tc {

using namespace cf::sm100;

constexpr int kPage = 16;
constexpr int HD = 128;                   // head dim (two 64-column swizzle atoms)
constexpr int kRows = 128;                // query rows per CTA (TMEM lanes)
constexpr int kKeys = 128;                // keys per block (8 pages)
constexpr int kStages = 3;                // K/V block ring (3 x 64 KB + Q 32 KB)
constexpr int kThreads = 11 * 32;
constexpr int kVWarp = 10;               // V producer warp
constexpr uint32_t kTileBytes = kKeys * HD * 2;  // 32 KB: one tensor, one block
constexpr uint32_t kBoxBytes = kKeys * 128;      // 16 KB: 64 columns of one block
constexpr uint32_t kQBytes = kRows * HD * 2;     // 32 KB
constexpr uint32_t kColS = 0, kColO = 256;  // S/P buffer g at 128 g, O of group g at 256 + 128 g
constexpr float kLazy = 8.0f;             // log2 headroom before the running max is raised
constexpr uint64_t kDrainNs = 1000000000ull;

struct Params {
  int B, R, G, Hkv, L, layer, rows_total, max_blocks;
  int64_t total_blocks;
  const __nv_bfloat16 *q;
  int64_t q_row_stride;
  const __nv_bfloat16 *k_new, *v_new;  // this layer: [B][R][Hkv][HD]
  const int32_t *block_tables, *context_lens;
  const uint64_t *tree_mask;
  int mask_words;
  __nv_bfloat16 *out;
  int64_t out_row_stride;
  float scale_log2;
  int *status;
  uint64_t timeout_ns;
  unsigned long long *trace;  // optional: [8][512] SM-clock stamps of CTA (0,0) per key block
};

__device__ __forceinline__ float ex2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-B chunk c (0..15) of row r in a [2 atoms][rows][128 B] tile with the
// 128-B swizzle (the layout TMA writes for two 64-column boxes, and tcgen05 reads).
__device__ __forceinline__ uint32_t sw_off(int r, int c, uint32_t atom_bytes) {
  return (uint32_t)((c >> 3) * atom_bytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
tree_attn_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                 const __grid_constant__ CUtensorMap tm_kn, const __grid_constant__ CUtensorMap tm_vn,
                 const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *q_s = smem;                                   // [2][128 rows][128 B]
  uint8_t *kv_s = smem + kQBytes;                        // [stage][K, V][2][128 keys][128 B]
  uint64_t *kv_full = reinterpret_cast<uint64_t *>(kv_s + kStages * 2 * kTileBytes);  // [K, V][stage]
  uint64_t *kv_empty = kv_full + 2 * kStages;  // K slot freed by QK_j, V slot by PV_j
  uint64_t *s_full = kv_empty + 2 * kStages;   // [2] QK_j done -> S buffer j%2 readable
  uint64_t *p_full = s_full + 2;           // [2] P_j in TMEM (the 4 warps of group j%2 arrive)
  uint64_t *o_done = p_full + 2;           // every MMA of the CTA done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_done + 1);
  volatile int &s_fail = *reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int b = blockIdx.y / p.Hkv, h = blockIdx.y % p.Hkv;
  const int ctx = p.context_lens[b];
  const int pc = (ctx + kPage - 1) / kPage;         // cached pages
  const int nc = (ctx + kKeys - 1) / kKeys;         // cached key blocks
  const int nb = nc + 1;                            // + the block of this step's new rows
  const int32_t *btab = p.block_tables + (int64_t)b * p.max_blocks;
  const bool tr = p.trace && blockIdx.x == 0 && blockIdx.y == 0;
#define CF_TTRACE(role, j) \
  if (tr && (j) < 512) p.trace[(role) * 512 + (j)] = clock64()
  if (tr && threadIdx.x == 0) p.trace[7 * 512] = clock64();

  // Q tile: row r = (new row rr, head-in-group g) with rr * G + g = tile * 128 + r
  for (int idx = threadIdx.x; idx < kRows * (HD / 8); idx += kThreads) {
    const int r = idx >> 4, c = idx & 15;
    const int qrow = tile * kRows + r;
    uint4 v = make_uint4(0, 0, 0, 0);  // rows past the group are zero
    if (qrow < p.rows_total) {
      const int rr = qrow / p.G, g = qrow % p.G;
      v = *reinterpret_cast<const uint4 *>(p.q + (int64_t)(b * p.R + rr) * p.q_row_stride +
                                           (int64_t)(h * p.G + g) * HD + c * 8);
    }
    *reinterpret_cast<uint4 *>(q_s + sw_off(r, c, kRows * 128)) = v;
  }
  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < 2 * kStages; ++s) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(&s_full[s], 1); mbar_init(&p_full[s], 4); }
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { prefetch_tmap(&tm_k); prefetch_tmap(&tm_v); prefetch_tmap(&tm_kn); prefetch_tmap(&tm_vn); }
  fence_proxy_async_smem();  // the Q tile (generic writes) -> async proxy
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued = 0;  // key blocks whose TMA loads this producer started (drained on failure)
  const int tv = warp == kVWarp ? 1 : 0;  // producer warps: the tensor they load

  if (warp == 0 || warp == kVWarp) {
    // ---------------- K (warp 0) / V (warp 10) producer ----------------
    const int pool_rows_per_block = p.L * p.Hkv * kPage;
    for (int j = 0; j < nb; ++j) {
      const int s = j % kStages;
      if (j >= kStages &&
          !mbar_wait_warp(&kv_empty[tv * kStages + s], (uint32_t)((j / kStages) & 1) ^ 1u, p.timeout_ns)) {
        ok = false;
        break;
      }
      uint8_t *ts = kv_s + s * 2 * kTileBytes + tv * kTileBytes;
      uint64_t *full = &kv_full[tv * kStages + s];
      if (j < nc) {
        const int p0 = j * (kKeys / kPage);
        // all 8 pages of the block: past the context the last cached page is loaded again,
        // so every key row holds finite values (their scores are masked; 0 x finite = 0)
        if (lane == 0) { if (tv == 0) CF_TTRACE(0, j); mbar_arrive_expect_tx(full, (uint32_t)kKeys * 2u * 128u); }
        __syncwarp();
        // 2 boxes per page (two 64-column halves), one per lane
        if (lane < 16) {
          const int pg = lane >> 1, bx = lane & 1;
          int blk = btab[min(p0 + pg, pc - 1)];
          if (blk < 0 || blk >= p.total_blocks) {  // invalid page id: record, read block 0
            if (p.status) atomicExch(p.status, CF_ERANGE);
            blk = 0;
          }
          const int y = blk * pool_rows_per_block + (p.layer * p.Hkv + h) * kPage;
          tma_load_2d(ts + bx * kBoxBytes + pg * (kPage * 128), tv ? &tm_v : &tm_k, full, bx * 64, y);
        }
        __syncwarp();
        issued = j + 1;
      } else {
        // this step's new rows: 128 rows from row b*R of the [B*R][Hkv][HD] scratch, head h
        // (rows past R belong to the next sequence or lie past the tensor, zero-filled; their
        // scores are masked), same swizzled layout as a block of pages
        if (lane == 0) { if (tv == 0) CF_TTRACE(0, j); mbar_arrive_expect_tx(full, 2u * kBoxBytes); }
        __syncwarp();
        if (lane < 2) tma_load_3d(ts + lane * kBoxBytes, tv ? &tm_vn : &tm_kn, full, lane * 64, h, b * p.R);
        __syncwarp();
        issued = j + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue (one thread) ----------------
    // QK_0, QK_1; then per block j: wait P_j, PV_j into O of group j%2, then QK_{j+2} into
    // S buffer j%2.  P_j lives in that buffer's first 64 columns; tcgen05.mma instructions of
    // one thread execute in issue order, so PV_j has read P_j before QK_{j+2} overwrites it.
    if (lane == 0) {
      const uint32_t id_qk = idesc_bf16_f32(kRows, kKeys);
      const uint32_t id_pv = idesc_bf16_f32(kRows, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t qa = smem_u32(q_s);
      auto qk = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&kv_full[s], (uint32_t)(j / kStages) & 1u, p.timeout_ns)) return false;  // K_j
        CF_TTRACE(1, j);
        tc_fence_after();
        const uint32_t kb = smem_u32(kv_s + s * 2 * kTileBytes);
        const uint32_t d = tmem + kColS + (uint32_t)(j & 1) * kKeys;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_f16(d, desc_kmajor_sw128(qa + (kk >> 2) * (kRows * 128) + (kk & 3) * 32),
                  desc_kmajor_sw128(kb + (kk >> 2) * kBoxBytes + (kk & 3) * 32), id_qk, kk > 0 ? 1u : 0u);
        mma_commit(&kv_empty[s]);  // K slot s free once QK_j has read it
        mma_commit(&s_full[j & 1]);
        return true;
      };
      ok = qk(0) && (nb < 2 || qk(1));
      for (int j = 0; ok && j < nb; ++j) {
        if (!mbar_wait(&p_full[j & 1], (uint32_t)(j >> 1) & 1u, p.timeout_ns)) { ok = false; break; }
        CF_TTRACE(2, j);
        const int s = j % kStages;
        if (!mbar_wait(&kv_full[kStages + s], (uint32_t)(j / kStages) & 1u, p.timeout_ns)) { ok = false; break; }  // V_j
        tc_fence_after();
        const uint32_t vb = smem_u32(kv_s + s * 2 * kTileBytes + kTileBytes);
        const uint32_t pa = tmem + kColS + (uint32_t)(j & 1) * kKeys;
        const uint32_t od = tmem + kColO + (uint32_t)(j & 1) * HD;
        // V block as the MN-major B operand: 16 keys (two 8-row groups, 1 KB apart) per MMA,
        // head dim in two 64-column atoms 16 KB apart
#pragma unroll
        for (int kt = 0; kt < kKeys / 16; ++kt)
          mma_f16_ts(od, pa + (uint32_t)(kt * 8), desc_mnmajor_sw128(vb + kt * 2048, kBoxBytes, 1024), id_pv,
                     (j >= 2 || kt > 0) ? 1u : 0u);
        mma_commit(&kv_empty[kStages + s]);
        if (j + 2 < nb && !qk(j + 2)) { ok = false; break; }
      }
      mma_commit(o_done);  // also on failure: completes once every issued MMA has finished
    }
    __syncwarp();
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  } else if (warp >= 2 && warp < kVWarp) {
    // ---------------- softmax: group g = (warp - 2) / 4 takes blocks j = g, g + 2, ... ----------------
    // one query row per thread; each group keeps its own running max m, sum l and O (TMEM),
    // merged at the end
    const int grp = (warp - 2) >> 2;
    const int qd = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t sa = tmem + lane_base + kColS + (uint32_t)grp * kKeys;  // S_j, then P_j in place
    const uint32_t oa = tmem + lane_base + kColO + (uint32_t)grp * HD;
    const int qrow = tile * kRows + row;
    const bool valid = qrow < p.rows_total;
    const int rq = valid ? qrow / p.G : 0;
    const float sl = p.scale_log2;
    // visibility of this step's new rows (keys of the last block) for this query row
    auto low_bits = [](int n, int w) -> uint64_t {  // bits j < n of word w
      const int k = n - 64 * w;
      return k <= 0 ? 0ull : (k >= 64 ? ~0ull : ((1ull << k) - 1ull));
    };
    uint64_t vis0 = 0, vis1 = 0;
    if (valid) {
      if (p.tree_mask) {
        const uint64_t *mw = p.tree_mask + ((int64_t)b * p.R + rq) * p.mask_words;
        vis0 = mw[0];
        vis1 = p.mask_words > 1 ? mw[1] : 0ull;
      } else {
        vis0 = low_bits(rq + 1, 0);
        vis1 = low_bits(rq + 1, 1);
      }
      vis0 &= low_bits(p.R, 0);
      vis1 &= low_bits(p.R, 1);
    }
    float m_used = -INFINITY, l = 0.0f;
    // a warp whose 32 rows are all past the group (the last row tile) only keeps the
    // barrier protocol: rows are independent in both products, and O rows past the group
    // are never written out, so whatever its P rows hold cannot reach a real row
    const bool warp_live = __any_sync(0xffffffffu, valid);
    for (int j = grp; j < nb; j += 2) {
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      // S_j ready; the commit also covers PV_{j-2}, so O of this group is current
      if (!mbar_wait_warp(&s_full[grp], ph, p.timeout_ns)) { ok = false; break; }
      if (threadIdx.x == 64) CF_TTRACE(3, j);
      if (!warp_live) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[grp]);
        continue;
      }
      tc_fence_after();
      const bool newblk = j == nc;
      // keep the per-key mask bits from being hoisted out of the block loop (128 live registers)
      asm volatile("" : "+l"(vis0), "+l"(vis1));
      const int kbase = j * kKeys;
      const bool full = !newblk && kbase + kKeys <= ctx;
      auto visible = [&](int col) -> bool {
        if (full) return true;
        if (newblk) return ((col < 64 ? vis0 >> col : vis1 >> (col - 64)) & 1ull) != 0;
        return kbase + col < ctx;
      };
      // pass 1: max of the visible raw scores, 64 columns at a time (two loads in flight)
      float mp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = -INFINITY;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t s0[32], s1[32];
        tmem_ld_32x32b_x32(sa + (uint32_t)(hf * 64), s0);
        tmem_ld_32x32b_x32(sa + (uint32_t)(hf * 64 + 32), s1);
        tmem_ld_wait();
        if (full) {  // the common case: no mask evaluation at all
#pragma unroll
          for (int e = 0; e < 64; ++e) mp[e & 7] = fmaxf(mp[e & 7], __uint_as_float(e < 32 ? s0[e] : s1[e - 32]));
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (visible(hf * 64 + e)) mp[e & 7] = fmaxf(mp[e & 7], __uint_as_float(e < 32 ? s0[e] : s1[e - 32]));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      // lazy running max: raise it (and rescale l and O) only when this block's max exceeds
      // it by more than kLazy in log2 units, or it is still -inf
      const float mb = mx * sl;
      const bool need = valid && mb != -INFINITY && (m_used == -INFINITY || mb > m_used + kLazy);
      const float f = need ? (m_used == -INFINITY ? 0.0f : ex2f_approx(m_used - mb)) : 1.0f;
      if (__any_sync(0xffffffffu, need)) {
        l *= f;
        if (j >= 2) {  // O of this group holds PV of its earlier blocks: scale this warp's rows
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(oa + (uint32_t)(c * 32), r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
            tmem_st_32x32b_x32(oa + (uint32_t)(c * 32), r);
          }
          tmem_st_wait();
        }
        if (need) m_used = mb;
      }
      if (threadIdx.x == 64) CF_TTRACE(5, j);
      // pass 2: P = 2^(s * scale * log2e - m) as bf16 pairs (keys 2i, 2i+1 per column),
      // written over the first 64 columns of this S buffer: chunk c (keys 32c..32c+31) is
      // read before columns 16c..16c+15 are written, and later chunks lie above them
      const bool live = m_used != -INFINITY;
      const float nm = live ? -m_used : 0.0f;
      float lp[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};  // partial sums
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(sa + (uint32_t)(c * 32), r);
        tmem_ld_wait();
        if (!full) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (!visible(c * 32 + e)) r[e] = __float_as_uint(-INFINITY);  // 2^-inf = 0
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = ex2f_approx(fmaf(__uint_as_float(r[e]), sl, nm));
          float p1 = ex2f_approx(fmaf(__uint_as_float(r[e + 1]), sl, nm));
          if (!live) p0 = p1 = 0.0f;
          lp[(e >> 1) & 7] += p0 + p1;
          pk[e >> 1] = pack_bf16(p0, p1);
        }
        tmem_st_32x32b_x16(sa + (uint32_t)(c * 16), pk);
      }
      l += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[grp]);
      if (threadIdx.x == 64) CF_TTRACE(4, j);
    }
    // ---------------- output: merge the two groups, O / l as bf16 ----------------
    if (!mbar_wait_warp(o_done, 0, ok ? p.timeout_ns : kDrainNs)) ok = false;
    tc_fence_after();
    // every MMA is done, so the Q tile is free: exchange (m, l) per row through it
    float *ml = reinterpret_cast<float *>(q_s);  // [group][m, l][128 rows]
    ml[grp * 256 + row] = m_used;
    ml[grp * 256 + 128 + row] = l;
    named_bar_sync(1, 8 * 32);  // the 8 softmax warps (all reach it: no early exit above)
    const float ma = ml[row], la = ml[128 + row], mbb = ml[256 + row], lb = ml[384 + row];
    const float M = fmaxf(ma, mbb);
    const float fa = (la > 0.0f && M != -INFINITY) ? ex2f_approx(ma - M) : 0.0f;
    const float fb = (lb > 0.0f && M != -INFINITY) ? ex2f_approx(mbb - M) : 0.0f;
    const float L = la * fa + lb * fb;
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    if (ok) {
      __nv_bfloat16 *dst = nullptr;
      if (valid) {
        const int g = qrow % p.G;
        dst = p.out + (int64_t)(b * p.R + rq) * p.out_row_stride + (int64_t)(h * p.G + g) * HD;
      }
      // group g writes head-dim columns [64 g, 64 g + 64) of its rows
      const uint32_t o0 = tmem + lane_base + kColO, o1 = o0 + HD;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = grp * 64 + c * 32;
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(o0 + (uint32_t)col, ra);
        tmem_ld_32x32b_x32(o1 + (uint32_t)col, rb);
        tmem_ld_wait();
        if (dst) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            // a group with no visible key contributes nothing (its O may be unwritten)
            const float v0 = (fa != 0.0f ? __uint_as_float(ra[2 * e]) * fa : 0.0f) +
                             (fb != 0.0f ? __uint_as_float(rb[2 * e]) * fb : 0.0f);
            const float v1 = (fa != 0.0f ? __uint_as_float(ra[2 * e + 1]) * fa : 0.0f) +
                             (fb != 0.0f ? __uint_as_float(rb[2 * e + 1]) * fb : 0.0f);
            w[e] = pack_bf16(v0 * inv, v1 * inv);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<uint4 *>(dst + col)[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
  }
  if (!ok) s_fail = 1;
  __syncthreads();
  if (s_fail) {
    // a wait ran out: let this CTA's own copies land and its MMAs finish (bounded) before
    // TMEM is freed and the CTA exits
    if (warp == 0 || warp == kVWarp) {
      for (int jj = max(0, issued - kStages); jj < issued; ++jj)
        mbar_wait_warp(&kv_full[tv * kStages + jj % kStages], (uint32_t)(jj / kStages) & 1u, kDrainNs);
    } else if (warp == 1) {
      mbar_wait_warp(o_done, 0, kDrainNs);
    }
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, CF_ETIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// Rows per kv head >= 128 (the warp-MMA kernel handles smaller groups), at most 128
// new rows, bf16, head dim 128, no explicit KV split requested.
bool eligible(const cf_attn_args &a) {
  if (a.kv.dtype != CF_BF16 || a.kv.head_dim != HD || a.kv.block_size != kPage) return false;
  const int G = a.num_q_heads / a.kv.num_kv_heads;
  return a.rows * G >= kRows && a.rows <= kKeys && a.num_splits <= 1 &&
         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
}

int launch(const cf_attn_args &a, cudaStream_t stream) {
  Params p;
  p.B = a.batch; p.R = a.rows; p.G = a.num_q_heads / a.kv.num_kv_heads; p.Hkv = a.kv.num_kv_heads;
  p.L = a.kv.num_layers; p.layer = a.layer;
  p.rows_total = a.rows * p.G;
  p.max_blocks = a.max_blocks; p.total_blocks = a.kv.total_blocks;
  p.q = reinterpret_cast<const __nv_bfloat16 *>(a.q); p.q_row_stride = a.q_row_stride;
  const int64_t layer_new = (int64_t)a.batch * a.rows * p.Hkv * HD;
  p.k_new = reinterpret_cast<const __nv_bfloat16 *>(a.k_new) + (a.new_kv_all_layers ? layer_new * a.layer : 0);
  p.v_new = reinterpret_cast<const __nv_bfloat16 *>(a.v_new) + (a.new_kv_all_layers ? layer_new * a.layer : 0);
  p.block_tables = a.block_tables; p.context_lens = a.context_lens;
  p.tree_mask = a.tree_mask; p.mask_words = a.mask_words;
  p.out = reinterpret_cast<__nv_bfloat16 *>(a.out); p.out_row_stride = a.out_row_stride;
  const float scale = a.scale > 0.0f ? a.scale : 1.0f / sqrtf((float)HD);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = a.status;
  p.timeout_ns = a.timeout_ns ? a.timeout_ns : 2000000000ull;
  p.trace = reinterpret_cast<unsigned long long *>(a.trace);
  const uint64_t pool_rows = (uint64_t)a.kv.total_blocks * p.L * p.Hkv * kPage;
  if (pool_rows > (uint64_t)INT32_MAX) return CF_EUNSUPPORTED;
  CUtensorMap tk, tv;
  if (!cf::make_tmap_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.kv.key_pool, HD, pool_rows, HD * 2, 64, kPage,
                        CU_TENSOR_MAP_SWIZZLE_128B) ||
      !cf::make_tmap_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.kv.val_pool, HD, pool_rows, HD * 2, 64, kPage,
                        CU_TENSOR_MAP_SWIZZLE_128B))
    return CF_EINVAL;
  CUtensorMap tkn, tvn;  // this step's new rows: [B*R][Hkv][HD], boxes of 128 rows x 64 columns of one head
  const uint64_t nrows = (uint64_t)a.batch * a.rows;
  if (!cf::make_tmap_3d(&tkn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.k_new, HD, p.Hkv, nrows, HD * 2,
                        (uint64_t)p.Hkv * HD * 2, 64, 1, kKeys, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !cf::make_tmap_3d(&tvn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.v_new, HD, p.Hkv, nrows, HD * 2,
                        (uint64_t)p.Hkv * HD * 2, 64, 1, kKeys, CU_TENSOR_MAP_SWIZZLE_128B))
    return CF_EINVAL;
  const size_t smem = 1024 + kQBytes + (size_t)kStages * 2 * kTileBytes + 256;
  CF_CUDA_TRY(cudaFuncSetAttribute(tree_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.rows_total + kRows - 1) / kRows, p.B * p.Hkv);
  tree_attn_kernel<<<grid, kThreads, smem, stream>>>(tk, tv, tkn, tvn, p);
  if (cudaGetLastError() != cudaSuccess) return CF_ECUDA;
  return cf_launch_status();
}

}  // namespace attn_tc
}  // namespace cf
