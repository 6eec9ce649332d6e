// Paged verify attention for speculative decoding (sm_100a).
//
// The R new query rows of each sequence (chain: the last emitted token + K
// drafts; tree: the root + N tree nodes) attend to
//   * the sequence's cached context, read page by page from the paged pool
//     [block][layer][kv_head][slot][head_dim] through TMA (two 64-column
//     boxes with 128-B swizzle per 16-token page per tensor), and
//   * the R new rows themselves (this step's K/V scratch), under a causal
//     (chain) or tree-ancestor mask.
// Semantics follow the reference's attention kernels (online softmax with
// scale head_dim^-1/2: csrc/kernels/triton/flash_attn_triton.py:7-110,
// csrc/kernels/cuda/flash_attn_v2.cu:46-195), extended with paging (the
// KVCacheBatchDescriptor contract, csrc/include/cudaforge/memory/
// paged_kv_cache.h:81-94), grouped-query heads and the tree mask.
//
// One CTA = (row tile of 16*NW query rows of one kv-head group) x (one KV
// split).  Query rows of a kv head are ordered (new row r, head-in-group g).
// Each warp owns 16 query rows; QK^T and PV use mma.sync m16n8k16 on
// ldmatrix fragments (K non-transposed, V transposed) with fp32 online
// softmax in registers.  The loop is HBM-bound (~24 FLOP per KV byte at
// GQA 4:1 and 6 rows), so the legacy warp MMA is ample; the pool stream is
// what the kernel is built around: an 8-slot TMA ring, 8 KB per page (HD 128).
// Several splits per sequence (flash-decoding) are merged by
// attn_combine_kernel in log-sum-exp form.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace cf {
namespace attn_tc {  // attention_tc.cu: tcgen05 path for >= 128 rows per kv head
bool eligible(const cf_attn_args &a);
int launch(const cf_attn_args &a, cudaStream_t stream);
}  // namespace attn_tc
}  // namespace cf

#include <algorithm>
#include <cstdlib>
#include <math.h>

namespace {

using namespace cf::sm100;

constexpr int kPage = 16;   // tokens per KV page (reference block_size 16)
constexpr uint64_t kDrainNs = 1000000000ull;

struct AttnParams {
  int B, R, G, Hkv, L, layer, rows_total, nsplit, max_blocks;
  int64_t total_blocks;
  const void *q;
  int64_t q_row_stride;
  const void *k_new, *v_new;  // this layer: [B][R][Hkv][D]
  const int32_t *block_tables, *context_lens;
  const uint64_t *tree_mask;
  int mask_words;
  void *out;
  int64_t out_row_stride;
  float scale_log2;
  float *ws_o, *ws_lse;
  int *status;
  uint64_t timeout_ns;
  unsigned long long *trace;
};

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <> struct MmaOp<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

// Hardware base-2 exponential (MUFU), flush-to-zero; ex2(-inf) = +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Byte offset of 16-B chunk `c` of row `r` in a KV page tile laid out as
// HD/64 boxes of [16 rows][128 B] with the TMA 128-B swizzle.
template <int HD>
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (uint32_t)((c >> 3) * (kPage * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
// Q tile: rows of HD*2 bytes, chunk index XOR (row & 7).
template <int HD>
__device__ __forceinline__ uint32_t q_off(int r, int c) {
  return (uint32_t)(r * (HD * 2) + ((c ^ (r & 7)) << 4));
}

// One CTA = 16*MTW query rows (one row tile of a kv-head group) x one KV
// split, run by kConsumers page streams of MTW warps each.  Page j of the
// split goes to stream j % 4; its ring slots are j % kStages (kStages is a
// multiple of 4, so a stream owns kStages / 4 slots).  The first warp of each
// stream is also that stream's loader: it fills the stream's slots ahead of
// use (each page's 64-column TMA boxes issued by a few of its lanes; the
// split's new-row tiles copied in with plain loads) and refills a slot once
// all MTW warps of the stream released it through the slot's `empty`
// barrier.  There is no separate producer warp: two 8-warp CTAs then fit on
// one SM at 128 registers per thread (four warps per SM sub-partition),
// enough for the online-softmax state without spilling.  Each warp keeps its
// own (m, l, O) over its 16 rows; the four streams' partial states are merged
// in shared memory at the end.
constexpr int kConsumers = 4;

template <int MTW>
constexpr int attn_min_ctas() { return MTW == 2 ? 2 : 3; }

template <typename T, int HD, int MTW, int kStages>
__global__ void __launch_bounds__(kConsumers * MTW * 32, attn_min_ctas<MTW>())
verify_attn_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                   const AttnParams p) {
  static_assert(kStages % kConsumers == 0, "each stream owns whole ring slots");
  constexpr int TILE_BYTES = kPage * HD * 2;  // one tensor, one page
  constexpr int CH = HD / 8;                  // 16-B chunks per row
  constexpr int NBOX = HD / 64;               // 64-column TMA boxes per tile
  constexpr int kRows = 16 * MTW;
  constexpr int MT = 1;  // m16 tiles per consumer warp
  constexpr int kThreadsAll = kConsumers * MTW * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *kv_s = smem;                                           // [stage][K, V]
  uint8_t *q_s = smem + kStages * 2 * TILE_BYTES;                 // [rows][HD]
  uint64_t *full = reinterpret_cast<uint64_t *>(q_s + kRows * HD * 2);
  uint64_t *empty = full + kStages;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row_tile = blockIdx.x;
  const int b = blockIdx.y / p.Hkv, h = blockIdx.y % p.Hkv;
  const int split = blockIdx.z;
  const int ctx = p.context_lens[b];
  const int pc = (ctx + kPage - 1) / kPage;  // cached pages
  const int pn = (p.R + kPage - 1) / kPage;  // new-row tiles
  const int T_all = pc + pn;
  const int tps = (T_all + p.nsplit - 1) / p.nsplit;
  const int t_begin = min(T_all, split * tps), t_end = min(T_all, t_begin + tps);
  const int ntiles = t_end - t_begin;
  const int32_t *btab = p.block_tables + (int64_t)b * p.max_blocks;
  const bool tr = p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  if (tr && tid == 0) p.trace[3072] = clock64();

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], MTW); }
    fence_mbar_init();
  }
  // ---- Q tile -> shared (rows >= R*G are zero) ----
  for (int idx = tid; idx < kRows * CH; idx += kThreadsAll) {
    const int r = idx / CH, c = idx % CH;
    const int qrow = row_tile * kRows + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (qrow < p.rows_total) {
      const int rr = qrow / p.G, g = qrow % p.G;
      const T *src = reinterpret_cast<const T *>(p.q) + (int64_t)(b * p.R + rr) * p.q_row_stride +
                     (int64_t)(h * p.G + g) * HD + c * 8;
      v = *reinterpret_cast<const uint4 *>(src);
    }
    *reinterpret_cast<uint4 *>(q_s + q_off<HD>(r, c)) = v;
  }
  __syncthreads();

  bool abort = false;
  float o[MT][HD / 8][4];
  float m_r[2 * MT], l_r[2 * MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) o[mt][d][0] = o[mt][d][1] = o[mt][d][2] = o[mt][d][3] = 0.0f;
#pragma unroll
  for (int hr = 0; hr < 2 * MT; ++hr) { m_r[hr] = -INFINITY; l_r[hr] = 0.0f; }

  const int cw = warp % kConsumers;            // page stream of this warp
  const int mrow0 = (warp / kConsumers) * 16;  // its m16 tile within the CTA rows
  const bool loader = mrow0 == 0;              // first warp of the stream fills its slots
  const int pool_rows_per_block = p.L * p.Hkv * kPage;
  // Fill ring slot j % kStages with tile j of this split (loader warp only).
  auto fill = [&](int j) {
    const int t = t_begin + j;
    const int s = j % kStages;
    uint8_t *st = kv_s + s * 2 * TILE_BYTES;
    if (tr && lane == 0 && j < 1024) p.trace[j] = clock64();
    if (t < pc) {
      int blk = btab[t];
      if (blk < 0 || blk >= p.total_blocks) {  // invalid page id: record and read page 0 (masked below)
        if (p.status && lane == 0) atomicExch(p.status, CF_ERANGE);
        blk = 0;
      }
      const int y = blk * pool_rows_per_block + (p.layer * p.Hkv + h) * kPage;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], 2 * TILE_BYTES);
      __syncwarp();
      if (lane < NBOX) tma_load_2d(st + lane * kPage * 128, &tm_k, &full[s], lane * 64, y);
      else if (lane < 2 * NBOX)
        tma_load_2d(st + TILE_BYTES + (lane - NBOX) * kPage * 128, &tm_v, &full[s], (lane - NBOX) * 64, y);
    } else {
      // new rows (t - pc)*16 ..: this step's K/V scratch rows (plain loads)
      const int j0 = (t - pc) * kPage;
      for (int idx = lane; idx < kPage * CH; idx += 32) {
        const int r = idx / CH, c = idx % CH;
        const int jr = j0 + r;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (jr < p.R) {
          const int64_t off = ((int64_t)(b * p.R + jr) * p.Hkv + h) * HD + c * 8;
          kv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const T *>(p.k_new) + off);
          vv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const T *>(p.v_new) + off);
        }
        *reinterpret_cast<uint4 *>(st + kv_off<HD>(r, c)) = kv;
        *reinterpret_cast<uint4 *>(st + TILE_BYTES + kv_off<HD>(r, c)) = vv;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);  // release: the rows are visible to the stream's warps
    }
  };
  int last_issued = cw - kConsumers;  // highest tile this loader has filled
  if (loader)
    for (int j = cw; j < min(ntiles, kStages); j += kConsumers) { fill(j); last_issued = j; }

  {
    // ---------------- consumers: page j goes to the MTW warps of stream j % 4 ----------------
    const uint32_t q_base = smem_u32(q_s);
    int pending_from = cw;  // first filled tile not yet known to have landed (drained on abort)
    for (int j = cw; j < ntiles; j += kConsumers) {
      const int t = t_begin + j;
      const int s = j % kStages;
      pending_from = j;
      if (!mbar_wait_warp_sleep(&full[s], (uint32_t)(j / kStages) & 1u, p.timeout_ns)) { abort = true; break; }
      if (tr && lane == 0 && mrow0 == 0 && j < 1024) p.trace[1024 + j] = clock64();
      const uint32_t k_base = smem_u32(kv_s + s * 2 * TILE_BYTES), v_base = k_base + TILE_BYTES;
      // S = Q K^T: rows x 16 tokens
      float sc[MT][2][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t kb[4];
        {
          const int tok = ((lane >> 4) << 3) + (lane & 7);
          const int c = 2 * kk + ((lane >> 3) & 1);
          ldsm_x4(k_base + kv_off<HD>(tok, c), kb);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t a[4];
          const int r = mrow0 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = 2 * kk + (lane >> 4);
          ldsm_x4(q_base + q_off<HD>(r, c), a);
          MmaOp<T>::run(sc[mt][0], a, kb[0], kb[1]);
          MmaOp<T>::run(sc[mt][1], a, kb[2], kb[3]);
        }
      }
      // mask (partial pages only) + online softmax in the log2 domain:
      // p = 2^(s * scale - m) with one FFMA + one hardware ex2 per element.
      const bool full_page = (t + 1) * kPage <= ctx;  // cached page with all 16 slots valid
      if (!full_page) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int col = nt * 8 + 2 * (lane & 3) + (e & 1);
              const int qrow = row_tile * kRows + mrow0 + mt * 16 + (lane >> 2) + (e >> 1) * 8;
              bool vis;
              if (t < pc) {
                vis = t * kPage + col < ctx;
              } else {
                const int jr = (t - pc) * kPage + col;
                const int rq = qrow / p.G;
                if (jr >= p.R || qrow >= p.rows_total) {
                  vis = false;
                } else if (p.tree_mask) {
                  const uint64_t w = p.tree_mask[((int64_t)b * p.R + rq) * p.mask_words + (jr >> 6)];
                  vis = (w >> (jr & 63)) & 1ull;
                } else {
                  vis = jr <= rq;
                }
              }
              if (!vis) sc[mt][nt][e] = -INFINITY;
            }
      }
      float mx[2 * MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const float raw = fmaxf(fmaxf(sc[mt][0][2 * e2], sc[mt][0][2 * e2 + 1]),
                                  fmaxf(sc[mt][1][2 * e2], sc[mt][1][2 * e2 + 1]));
          mx[mt * 2 + e2] = raw;
        }
#pragma unroll
      for (int hr = 0; hr < 2 * MT; ++hr) {
        mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
        mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
        mx[hr] = fmaxf(m_r[hr], mx[hr] * p.scale_log2);  // new running max (log2 units)
      }
      float corr[2 * MT];
      bool moved = false;
#pragma unroll
      for (int hr = 0; hr < 2 * MT; ++hr) {
        corr[hr] = (mx[hr] == m_r[hr]) ? 1.0f : ex2_approx(m_r[hr] - mx[hr]);  // -inf - x -> 0
        moved |= mx[hr] != m_r[hr];
        m_r[hr] = mx[hr];
        l_r[hr] *= corr[hr];
      }
      uint32_t pa[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float pv[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hr = mt * 2 + (e >> 1);
            // a row that has seen only masked keys keeps m = -inf: its p must be 0
            const float pe = (m_r[hr] == -INFINITY) ? 0.0f
                                                    : ex2_approx(fmaf(sc[mt][nt][e], p.scale_log2, -m_r[hr]));
            pv[nt][e] = pe;
            l_r[hr] += pe;
          }
        pa[mt][0] = MmaOp<T>::pack(pv[0][0], pv[0][1]);
        pa[mt][1] = MmaOp<T>::pack(pv[0][2], pv[0][3]);
        pa[mt][2] = MmaOp<T>::pack(pv[1][0], pv[1][1]);
        pa[mt][3] = MmaOp<T>::pack(pv[1][2], pv[1][3]);
      }
      // rescale O only when some row's running max moved (rare after the first pages)
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int d = 0; d < HD / 8; ++d) {
            o[mt][d][0] *= corr[mt * 2]; o[mt][d][1] *= corr[mt * 2];
            o[mt][d][2] *= corr[mt * 2 + 1]; o[mt][d][3] *= corr[mt * 2 + 1];
          }
      }
      // O += P V
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t vb[4];
        const int tok = (((lane >> 3) & 1) << 3) + (lane & 7);
        const int c = 2 * dp + (lane >> 4);
        ldsm_x4_t(v_base + kv_off<HD>(tok, c), vb);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          MmaOp<T>::run(o[mt][2 * dp], pa[mt], vb[0], vb[1]);
          MmaOp<T>::run(o[mt][2 * dp + 1], pa[mt], vb[2], vb[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // slot s may be refilled
      if (tr && lane == 0 && mrow0 == 0 && j < 1024) p.trace[2048 + j] = clock64();
      if (loader && j + kStages < ntiles) {
        // every warp of the stream is done with tile j: refill its slot with tile j + kStages
        pending_from = j + kConsumers;
        if (!mbar_wait_warp_sleep(&empty[s], (uint32_t)(j / kStages) & 1u, p.timeout_ns)) { abort = true; break; }
        fill(j + kStages);
        last_issued = j + kStages;
      }
    }
    if (abort && loader)  // let this warp's own copies land before the CTA can exit
      for (int jj = pending_from; jj <= last_issued; jj += kConsumers)
        if (t_begin + jj < pc) mbar_wait_warp(&full[jj % kStages], (uint32_t)(jj / kStages) & 1u, kDrainNs);
  }
  if (abort && p.status && lane == 0) atomicExch(p.status, CF_ETIMEOUT);
  const int any_abort = __syncthreads_or(abort ? 1 : 0);
  if (tr && tid == 0) p.trace[3073] = clock64();
  // ---- merge the consumers' (m, l, O) per row in shared memory ----
#pragma unroll
  for (int hr = 0; hr < 2 * MT; ++hr) {
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
  }
  float *so = reinterpret_cast<float *>(kv_s);            // [stream][rows][HD]
  float *sm_ = so + kConsumers * kRows * HD;                // [stream][rows]
  float *sl = sm_ + kConsumers * kRows;                     // [stream][rows]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int r = mrow0 + mt * 16 + (lane >> 2) + e2 * 8;
      float *dst = so + (cw * kRows + r) * HD;
#pragma unroll
      for (int d = 0; d < HD / 8; ++d)
        *reinterpret_cast<float2 *>(dst + d * 8 + 2 * (lane & 3)) = make_float2(o[mt][d][2 * e2], o[mt][d][2 * e2 + 1]);
      if ((lane & 3) == 0) { sm_[cw * kRows + r] = abort ? -INFINITY : m_r[mt * 2 + e2]; sl[cw * kRows + r] = l_r[mt * 2 + e2]; }
    }
  __syncthreads();
  if (any_abort) return;
  for (int idx = tid; idx < kRows * HD; idx += kThreadsAll) {
    const int r = idx / HD, d = idx % HD;
    const int qrow = row_tile * kRows + r;
    if (qrow >= p.rows_total) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, sm_[w * kRows + r]);
    float num = 0.0f, den = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float mw = sm_[w * kRows + r];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - M);
        num += f * so[(w * kRows + r) * HD + d];
        den += f * sl[w * kRows + r];
      }
    }
    const int rr = qrow / p.G, g = qrow % p.G;
    if (p.nsplit == 1) {
      T *dst = reinterpret_cast<T *>(p.out) + (int64_t)(b * p.R + rr) * p.out_row_stride + (int64_t)(h * p.G + g) * HD;
      const float v = den > 0.0f ? num / den : 0.0f;
      if constexpr (std::is_same<T, __half>::value) dst[d] = __float2half_rn(v);
      else dst[d] = __float2bfloat16_rn(v);
    } else {
      const int64_t rowid = (((int64_t)split * p.B + b) * p.Hkv + h) * p.rows_total + qrow;
      p.ws_o[rowid * HD + d] = den > 0.0f ? num / den : 0.0f;
      if (d == 0) p.ws_lse[rowid] = den > 0.0f ? M + log2f(den) : -INFINITY;
    }
  }
}

// Merge the per-split partial outputs (normalised O_s, lse_s in log2 units).
template <typename T, int HD>
__global__ void attn_combine_kernel(const AttnParams p) {
  const int bh = blockIdx.x, qrow = blockIdx.y;
  const int b = bh / p.Hkv, h = bh % p.Hkv;
  const int64_t stride = (int64_t)p.B * p.Hkv * p.rows_total;
  const int64_t base = ((int64_t)b * p.Hkv + h) * p.rows_total + qrow;
  float mx = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) mx = fmaxf(mx, p.ws_lse[s * stride + base]);
  const int rr = qrow / p.G, g = qrow % p.G;
  T *dst = reinterpret_cast<T *>(p.out) + (int64_t)(b * p.R + rr) * p.out_row_stride + (int64_t)(h * p.G + g) * HD;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float num = 0.0f, den = 0.0f;
    for (int s = 0; s < p.nsplit; ++s) {
      const float l = p.ws_lse[s * stride + base];
      if (l == -INFINITY) continue;
      const float w = exp2f(l - mx);
      num += w * p.ws_o[(s * stride + base) * HD + d];
      den += w;
    }
    const float v = den > 0.0f ? num / den : 0.0f;
    if constexpr (std::is_same<T, __half>::value) dst[d] = __float2half_rn(v);
    else dst[d] = __float2bfloat16_rn(v);
  }
}

// Row tiles of 16 query rows per page stream: 1 when a kv-head group's rows fit
// in 16 (decode-like steps: fewer idle MMA rows, up to three CTAs per SM), else 2.
int attn_mt(int rows_total) {
  return rows_total <= 16 ? 1 : 2;
}

int pick_splits(const cf_attn_args &a, int row_tiles, int per_sm) {
  if (a.num_splits > 0) return a.num_splits;
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ctas = a.batch * a.kv.num_kv_heads * row_tiles;
  // per_sm resident CTAs per SM: split the context only when the grid would not fill them
  const int want = ctas >= per_sm * sms ? 1 : (per_sm * sms + ctas - 1) / ctas;
  const int pages = (a.max_context + kPage - 1) / kPage;
  return std::max(1, std::min(want, std::max(1, pages / 8)));
}

template <typename T, int HD, int MT, int kStages>
int launch(const cf_attn_args &a, cudaStream_t stream) {
  constexpr int ROWS = 16 * MT;
  const int G = a.num_q_heads / a.kv.num_kv_heads;
  AttnParams p;
  p.B = a.batch; p.R = a.rows; p.G = G; p.Hkv = a.kv.num_kv_heads; p.L = a.kv.num_layers; p.layer = a.layer;
  p.rows_total = a.rows * G;
  const int row_tiles = (p.rows_total + ROWS - 1) / ROWS;
  p.nsplit = pick_splits(a, row_tiles, attn_min_ctas<MT>());
  p.max_blocks = a.max_blocks; p.total_blocks = a.kv.total_blocks;
  p.q = a.q; p.q_row_stride = a.q_row_stride;
  const int64_t layer_new = (int64_t)a.batch * a.rows * p.Hkv * HD;
  p.k_new = reinterpret_cast<const T *>(a.k_new) + (a.new_kv_all_layers ? layer_new * a.layer : 0);
  p.v_new = reinterpret_cast<const T *>(a.v_new) + (a.new_kv_all_layers ? layer_new * a.layer : 0);
  p.block_tables = a.block_tables; p.context_lens = a.context_lens;
  p.tree_mask = a.tree_mask; p.mask_words = a.mask_words;
  p.out = a.out; p.out_row_stride = a.out_row_stride;
  const float scale = a.scale > 0.0f ? a.scale : 1.0f / sqrtf((float)HD);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = a.status;
  p.timeout_ns = a.timeout_ns ? a.timeout_ns : 2000000000ull;
  p.trace = reinterpret_cast<unsigned long long *>(a.trace);
  if (p.nsplit > 1) {
    const size_t rows = (size_t)p.nsplit * p.B * p.Hkv * p.rows_total;
    const size_t need = rows * HD * sizeof(float) + rows * sizeof(float);
    if (!a.workspace || a.workspace_bytes < need || (reinterpret_cast<uintptr_t>(a.workspace) & 15)) return CF_EINVAL;
    p.ws_o = reinterpret_cast<float *>(a.workspace);
    p.ws_lse = p.ws_o + rows * HD;
  } else {
    p.ws_o = p.ws_lse = nullptr;
  }
  const CUtensorMapDataType tdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t pool_rows = (uint64_t)a.kv.total_blocks * p.L * p.Hkv * kPage;
  if (pool_rows > (uint64_t)INT32_MAX) return CF_EUNSUPPORTED;
  CUtensorMap tk, tv;
  if (!cf::make_tmap_2d(&tk, tdt, a.kv.key_pool, HD, pool_rows, HD * 2, 64, kPage, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !cf::make_tmap_2d(&tv, tdt, a.kv.val_pool, HD, pool_rows, HD * 2, 64, kPage, CU_TENSOR_MAP_SWIZZLE_128B))
    return CF_EINVAL;
  // the stage area is reused for the merge: [4][rows][HD] fp32 + m, l
  const size_t stage_area = std::max<size_t>((size_t)kStages * 2 * kPage * HD * 2,
                                             (size_t)kConsumers * ROWS * (HD + 2) * 4);
  const size_t smem = 1024 + stage_area + ROWS * HD * 2 + kStages * 16;
  auto kern = verify_attn_kernel<T, HD, MT, kStages>;
  CF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  dim3 grid(row_tiles, p.B * p.Hkv, p.nsplit);
  kern<<<grid, kConsumers * MT * 32, smem, stream>>>(tk, tv, p);
  if (cudaGetLastError() != cudaSuccess) return CF_ECUDA;
  if (p.nsplit > 1) {
    dim3 g2(p.B * p.Hkv, p.rows_total);
    attn_combine_kernel<T, HD><<<g2, HD / 2 >= 32 ? HD / 2 : 32, 0, stream>>>(p);
  }
  return cf_launch_status();
}

template <typename T>
int dispatch(const cf_attn_args &a, cudaStream_t s) {
  const int mt = attn_mt(a.rows * (a.num_q_heads / a.kv.num_kv_heads));
  if (a.kv.head_dim == 128) return mt == 2 ? launch<T, 128, 2, 8>(a, s) : launch<T, 128, 1, 8>(a, s);
  if (a.kv.head_dim == 64) return mt == 2 ? launch<T, 64, 2, 8>(a, s) : launch<T, 64, 1, 8>(a, s);
  return CF_EUNSUPPORTED;
}

}  // namespace

extern "C" size_t cf_attention_workspace_bytes(const cf_attn_args *a) {
  if (!a || a->kv.num_kv_heads <= 0 || a->num_q_heads % a->kv.num_kv_heads) return 0;
  if (cf::attn_tc::eligible(*a)) return 0;
  const int G = a->num_q_heads / a->kv.num_kv_heads;
  const int rows_total = a->rows * G;
  const int mt = attn_mt(rows_total);
  const int ROWS = 16 * mt;
  const int nsplit = pick_splits(*a, (rows_total + ROWS - 1) / ROWS, mt == 2 ? attn_min_ctas<2>() : attn_min_ctas<1>());
  if (nsplit <= 1) return 0;
  const size_t rows = (size_t)nsplit * a->batch * a->kv.num_kv_heads * rows_total;
  return rows * a->kv.head_dim * sizeof(float) + rows * sizeof(float);
}

extern "C" int cf_verify_attention(const cf_attn_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  const cf_attn_args &a = *args;
  if (a.batch < 0 || a.rows <= 0 || a.kv.num_kv_heads <= 0 || a.num_q_heads % a.kv.num_kv_heads) return CF_EINVAL;
  if (a.batch == 0) return CF_OK;
  if (a.kv.block_size != kPage || a.layer < 0 || a.layer >= a.kv.num_layers) return CF_EINVAL;
  if (!a.q || !a.k_new || !a.v_new || !a.block_tables || !a.context_lens || !a.out) return CF_EINVAL;
  if (!a.kv.key_pool || !a.kv.val_pool || a.kv.total_blocks <= 0) return CF_EINVAL;
  if (a.tree_mask && a.mask_words * 64 < a.rows) return CF_EINVAL;
  if ((a.q_row_stride % 8) || (a.out_row_stride % 8) || (reinterpret_cast<uintptr_t>(a.q) & 15) ||
      (reinterpret_cast<uintptr_t>(a.k_new) & 15) || (reinterpret_cast<uintptr_t>(a.v_new) & 15))
    return CF_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cf::attn_tc::eligible(a)) return cf::attn_tc::launch(a, s);
  if (a.kv.dtype == CF_BF16) return dispatch<__nv_bfloat16>(a, s);
  if (a.kv.dtype == CF_F16) return dispatch<__half>(a, s);
  return CF_EUNSUPPORTED;
}
