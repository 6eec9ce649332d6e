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
//   the MMA computes D^T[n, m] = W[n, :] . X[m, :]; the weight tile
//   (128 n x 64 k) is the tcgen05 "A" operand and the token tile (up to 512
//   tokens x 64 k, in <= 256-token MMA chunks) the "B" operand, so every
//   dequantised weight element feeds up to 512 tokens.  One CTA = one
//   128-row weight tile x one K split x one token slice; 6 warps:
//     warp 0      TMA producer (packed weights, group scales, token tile)
//     warp 1      TMEM allocator + the single MMA-issuing thread
//     warps 2-5   INT4 -> bf16 dequantisation into the 128-B swizzled A tile,
//                 then the epilogue (tcgen05.ld from TMEM -> global)
//   Every mbarrier wait is bounded (a device status word records CF_ETIMEOUT).
//   No TMA multicast is used.
//
// The packed weights are consumed in a kernel-native nibble order produced
// once per weight by cf_w4a16_repack (the same values; see dequant8()).
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

#include <algorithm>

namespace {

using namespace cf::sm100;

constexpr int kThreads = 192;
constexpr int BN = 128;  // weight rows per CTA (MMA M)
constexpr int BK = 64;   // k per pipeline stage: one 128-B swizzle atom of 16-bit elements
constexpr int kMaxSlice = 512;
constexpr int kMaxSmem = 232448;
constexpr uint32_t kATileBytes = BN * BK * 2;  // 16 KB
constexpr uint32_t kWPackBytes = (BK / 8) * BN * 4;  // 4 KB
constexpr uint32_t kScaleBytes = BN * 2;
constexpr uint64_t kDrainNs = 1000000000ull;

enum WMode : int { kInt4 = 0, kDense = 1 };

struct GemmParams {
  int M, N, K;
  int m_slice, chunks, chunk_rows, stages, kb_per_split, splits;
  uint32_t stage_bytes, off_x, off_w, off_s;
  uint32_t tmem_cols, idesc;
  void *y;
  int64_t ldy;
  const void *residual;
  int64_t ldr;
  float *partial;
  int *status;
  uint64_t timeout_ns;
};

// 8 repacked nibbles -> 8 bf16 (k order 0..7).  Repacked nibble position p
// holds k = 2p for p < 4 and k = 2(p-4)+1 for p >= 4, so masking with
// 0x000F000F after shifts of 0/4/8/12 yields the pairs (k0,k1) (k2,k3)
// (k4,k5) (k6,k7).  OR-ing 0x4300 builds bf16 128 + nibble exactly;
// subtracting 136 gives nibble - 8 exactly; one bf16 multiply by the scale.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __nv_bfloat162 s2) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u;
  const __nv_bfloat162 k136 = __floats2bfloat162_rn(136.0f, 136.0f);
  uint32_t h[4] = {(w & kMask) | kMagic, ((w >> 4) & kMask) | kMagic, ((w >> 8) & kMask) | kMagic,
                   ((w >> 12) & kMask) | kMagic};
  uint4 o;
  uint32_t *op = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&h[j]);
    v = __hmul2(__hsub2(v, k136), s2);
    op[j] = *reinterpret_cast<uint32_t *>(&v);
  }
  return o;
}

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T, int WM>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
            const __grid_constant__ CUtensorMap tm_s, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * p.stage_bytes);
  uint64_t *deq = full + S;
  uint64_t *empty = deq + S;
  uint64_t *accf = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int split = blockIdx.y;
  const int m0 = blockIdx.z * p.m_slice;
  const int mrows = min(p.m_slice, p.M - m0);
  const int kbs = p.K / BK;
  const int kb0 = split * p.kb_per_split;
  const int nkb = min(p.kb_per_split, kbs - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], 4);
      mbar_init(&empty[s], 1);
    }
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

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint32_t x_bytes = (uint32_t)(p.chunks * p.chunk_rows) * 128u;
      const uint32_t bytes = x_bytes + (WM == kInt4 ? kWPackBytes + kScaleBytes : kATileBytes);
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (i >= S && !mbar_wait(&empty[s], ph ^ 1u, p.timeout_ns)) { ok = false; break; }
        uint8_t *st = smem + s * p.stage_bytes;
        const int kb = kb0 + i;
        mbar_arrive_expect_tx(&full[s], bytes);
        for (int j = 0; j < p.chunks; ++j)
          tma_load_2d(st + p.off_x + j * p.chunk_rows * 128, &tm_x, &full[s], kb * BK, m0 + j * p.chunk_rows);
        if (WM == kInt4) {
          tma_load_2d(st + p.off_w, &tm_w, &full[s], n0, kb * (BK / 8));
          tma_load_2d(st + p.off_s, &tm_s, &full[s], n0, (kb * BK) / 128);
        } else {
          tma_load_2d(st, &tm_w, &full[s], kb * BK, n0);
        }
        issued = i + 1;
      }
      if (!ok) {  // let our own copies land before the CTA can exit
        for (int j = max(0, issued - S); j < issued; ++j)
          mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, kDrainNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- single MMA-issuing thread ----------------
      const uint32_t idesc = p.idesc;
      int i = 0;
      for (; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&full[s], ph, p.timeout_ns)) { ok = false; break; }
        if (WM == kInt4 && !mbar_wait(&deq[s], ph, p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + s * p.stage_bytes);
        const uint32_t x_base = a_base + p.off_x;
#pragma unroll
        for (int k16 = 0; k16 < BK / 16; ++k16) {
          const uint64_t ad = desc_kmajor_sw128(a_base + k16 * 32);
          for (int j = 0; j < p.chunks; ++j) {
            const uint64_t bd = desc_kmajor_sw128(x_base + j * p.chunk_rows * 128 + k16 * 32);
            mma_f16(tmem + (uint32_t)(j * p.chunk_rows), ad, bd, idesc, (i > 0 || k16 > 0) ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
      }
      mma_commit(accf);  // completes when every issued MMA has finished
    }
  } else {
    // ---------------- dequantisation (warps 2-5) ----------------
    const int t = threadIdx.x - 64;  // weight row within the tile
    if (WM == kInt4) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&full[s], ph, p.timeout_ns)) { ok = false; break; }
        uint8_t *st = smem + s * p.stage_bytes;
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(st + p.off_w);
        const __half sc = reinterpret_cast<const __half *>(st + p.off_s)[t];
        const __nv_bfloat16 sb = __float2bfloat16_rn(__half2float(sc));
        const __nv_bfloat162 s2 = __halves2bfloat162(sb, sb);
        uint8_t *arow = st + t * 128;
        uint32_t w[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) w[kk] = wp[kk * BN + t];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          *reinterpret_cast<uint4 *>(arow + ((kk ^ (t & 7)) << 4)) = dequant8(w[kk], s2);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
      }
    }
    // ---------------- epilogue ----------------
    if (!mbar_wait(accf, 0, ok ? p.timeout_ns : kDrainNs)) ok = false;
    tc_fence_after();
    if (ok) {
      const int q = warp & 3;  // TMEM lane quarter this warp may access
      const int n = n0 + q * 32 + lane;
      T *y = reinterpret_cast<T *>(p.y);
      const T *res = reinterpret_cast<const T *>(p.residual);
      for (int c = 0; c < mrows; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
        tmem_ld_wait();
        const int lim = min(32, mrows - c);
        if (p.splits > 1) {
          float *dst = p.partial + ((int64_t)split * p.M + (m0 + c)) * p.N + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < lim) dst[(int64_t)j * p.N] = __uint_as_float(r[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < lim) {
              const int64_t m = m0 + c + j;
              float v = __uint_as_float(r[j]);
              if (res) v += cf::to_float(res[m * p.ldr + n]);
              y[m * p.ldy + n] = from_f<T>(v);
            }
          }
        }
      }
    }
  }
  if (!ok && p.status) atomicExch(p.status, CF_ETIMEOUT);
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
  int slices, m_slice, chunks, chunk_rows, stages, splits, kb_per_split;
  uint32_t stage_bytes, off_x, off_w, off_s, tmem_cols;
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
  pl.slices = (M + kMaxSlice - 1) / kMaxSlice;
  const int per = (M + pl.slices - 1) / pl.slices;
  pl.chunks = (per + 255) / 256;
  pl.chunk_rows = ((per + pl.chunks - 1) / pl.chunks + 15) / 16 * 16;
  pl.m_slice = pl.chunks * pl.chunk_rows;
  if (pl.m_slice > kMaxSlice) return false;
  pl.off_x = kATileBytes;
  pl.off_w = pl.off_x + (uint32_t)pl.m_slice * 128u;
  pl.off_s = pl.off_w + (int4 ? kWPackBytes : 0);
  pl.stage_bytes = (pl.off_s + (int4 ? kScaleBytes : 0) + 1023u) & ~1023u;
  const size_t fixed = 1024 + 1024;  // alignment slack + barriers
  pl.stages = (int)std::min<size_t>(6, (kMaxSmem - fixed) / pl.stage_bytes);
  if (pl.stages < 2) return false;
  pl.smem = fixed + (size_t)pl.stages * pl.stage_bytes;
  uint32_t cols = 32;
  while (cols < (uint32_t)pl.m_slice) cols <<= 1;
  pl.tmem_cols = cols;
  const int kbs = K / BK;
  const int tiles = (N / BN) * pl.slices;
  int splits = split_req > 0 ? split_req : std::max(1, num_sms() / tiles);
  splits = std::max(1, std::min(splits, kbs / 2 > 0 ? kbs / 2 : 1));
  pl.kb_per_split = (kbs + splits - 1) / splits;
  pl.splits = (kbs + pl.kb_per_split - 1) / pl.kb_per_split;
  return true;
}

template <typename T, int WM>
int run_gemm(const cf_gemm_args &a, cudaStream_t stream) {
  const bool int4 = WM == kInt4;
  if (a.m < 0 || a.n <= 0 || a.k <= 0) return CF_EINVAL;
  if (a.m == 0) return CF_OK;
  if (a.n % BN != 0 || a.k % (int4 ? 128 : BK) != 0) return CF_EINVAL;
  if (!a.x || !a.w || !a.y || (int4 && !a.scales)) return CF_EINVAL;
  if (a.ldx < a.k || a.ldy < a.n || (a.residual && a.ldr < a.n)) return CF_EINVAL;
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
  if (!cf::make_tmap_2d(&tx, tdt, a.x, (uint64_t)a.k, (uint64_t)a.m, (uint64_t)a.ldx * 2, BK, pl.chunk_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B))
    return CF_EINVAL;
  if (int4) {
    if (!cf::make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, (uint64_t)a.n, (uint64_t)a.k / 8,
                          (uint64_t)a.n * 4, BN, BK / 8, CU_TENSOR_MAP_SWIZZLE_NONE))
      return CF_EINVAL;
    if (!cf::make_tmap_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.scales, (uint64_t)a.n, (uint64_t)a.k / 128,
                          (uint64_t)a.n * 2, BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return CF_EINVAL;
  } else {
    if (!cf::make_tmap_2d(&tw, tdt, a.w, (uint64_t)a.k, (uint64_t)a.n, (uint64_t)a.k * 2, BK, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return CF_EINVAL;
    ts = tw;
  }
  GemmParams p;
  p.M = a.m; p.N = a.n; p.K = a.k;
  p.m_slice = pl.m_slice; p.chunks = pl.chunks; p.chunk_rows = pl.chunk_rows; p.stages = pl.stages;
  p.kb_per_split = pl.kb_per_split; p.splits = pl.splits;
  p.stage_bytes = pl.stage_bytes; p.off_x = pl.off_x; p.off_w = pl.off_w; p.off_s = pl.off_s;
  p.tmem_cols = pl.tmem_cols;
  p.idesc = cf::sm100::idesc_bf16_f32(BN, pl.chunk_rows);
  if (std::is_same<T, __half>::value) p.idesc &= ~((7u << 7) | (7u << 10));  // A, B format f16
  p.y = a.y; p.ldy = a.ldy; p.residual = a.residual; p.ldr = a.ldr;
  p.partial = reinterpret_cast<float *>(a.workspace);
  p.status = a.status;
  p.timeout_ns = a.timeout_ns ? a.timeout_ns : 2000000000ull;
  auto kern = gemm_kernel<T, WM>;
  CF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
  dim3 grid(a.n / BN, pl.splits, pl.slices);
  kern<<<grid, kThreads, pl.smem, stream>>>(tx, tw, ts, p);
  if (cudaGetLastError() != cudaSuccess) return CF_ECUDA;
  if (pl.splits > 1) {
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

extern "C" int cf_w4a16_repack(const uint32_t *wq_ref, uint32_t *wq_out, int32_t k, int32_t n, void *stream) {
  if (!wq_ref || !wq_out || k <= 0 || n <= 0 || k % 8 != 0) return CF_EINVAL;
  const int64_t words = (int64_t)(k / 8) * n;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 4096);
  repack_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(wq_ref, wq_out, words);
  return cf_launch_status();
}
