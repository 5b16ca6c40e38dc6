// tcgen05 GEMM for sm_100a: TMA -> shared memory (128-byte swizzle) -> tcgen05.mma (fp32 accumulators in TMEM)
// -> tcgen05.ld epilogue with the MLP's fused elementwise work.
//
// One CTA computes one 128 x BN output tile (split-K partials along blockIdx.z). Warp roles:
//   warp 0      : TMA producer (one elected lane), multi-stage ring of shared-memory stages
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..9  : epilogue; warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32) = output rows of its quadrant, the two
//                 warps of a quadrant splitting the column chunks
// Short-K layers run two CTAs per SM (TMEM 2 x BN <= 512 columns) so that one CTA's epilogue overlaps the other's
// main loop.
// No load uses cluster multicast: every CTA fetches its own tiles from this GPU's memory.
//
// The MLP layers of rsl_rl (rsl_rl/modules/mlp.py:91-95, Linear+ELU stacks) map onto three uses:
//   forward : H_l   = elu(H_{l-1} W_l^T + b_l)      A = H_{l-1} (K-major), B = W_l (K-major)
//   dgrad   : dZ_l  = (dZ_{l+1} W_{l+1}) * elu'(H_l) A = dZ_{l+1} (K-major), B = W_{l+1} read MN-major
//   wgrad   : dW_l  = dZ_l^T H_{l-1}                A = dZ_l (MN-major), B = H_{l-1} (MN-major), split-K partials
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "gemm_tcgen05.cuh"
#include "sm100_primitives.cuh"

namespace rlb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle atom row
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quadrant, splitting the column chunks
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMNBoxBytes = 64 * kBK * 2;  // one {64 MN x 64 K} box
constexpr int kStageWords = 32 * 33;       // per-warp 32 x 32-word staging tile (+1 word padding per row)

template <int BN, int EPI>
struct Cfg {
  // Short-K layers (forward, data gradient) keep two CTAs per SM so one CTA's epilogue overlaps the other's
  // main loop; the long-K weight-gradient GEMM uses a deeper pipeline with one CTA per SM.
  static constexpr bool kLongK = EPI == kEpiPartialF32;
  static constexpr int kStages = kLongK ? (BN == 256 ? 4 : 6) : (BN == 256 ? 2 : BN == 128 ? 3 : 4);
  static constexpr int kMinBlocks = kLongK ? 1 : 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kColsumBytes = 4 * BN * 4;
  static constexpr int kPipeBytes = kStages * (kABytes + kBBytes);
  static constexpr int kSmemBytes = 1024 /*alignment slack*/ + kPipeBytes + kBarrierBytes + kColsumBytes;
  static_assert(kPipeBytes >= kEpiWarps * 2 * kStageWords * 4, "epilogue staging must fit in the pipeline buffers");
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, Cfg<BN, EPI>::kMinBlocks)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p, int num_kb) {
  using C = Cfg<BN, EPI>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * C::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* colsum_s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + C::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * BN;
  const int splits = gridDim.z;
  const int kb_begin = static_cast<int>((static_cast<long long>(blockIdx.z) * num_kb) / splits);
  const int kb_end = static_cast<int>((static_cast<long long>(blockIdx.z + 1) * num_kb) / splits);
  const int nkb = kb_end - kb_begin;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          report_error(p.status, kTimeoutSmemEmpty, 1);
          break;
        }
        const int kc = (kb_begin + i) * kBK;
        uint32_t bytes = 0;
        if (!A_MN) {
          bytes += kABytes;
        } else {
#pragma unroll
          for (int j = 0; j < kBM / 64; ++j)
            if (m0 + 64 * j < p.M) bytes += kMNBoxBytes;
        }
        if (!B_MN) {
          bytes += C::kBBytes;
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            if (n0 + 64 * j < p.N) bytes += kMNBoxBytes;
        }
        mbar_arrive_expect_tx(&full[s], bytes);
        uint8_t* a_dst = sA + s * kABytes;
        uint8_t* b_dst = sB + s * C::kBBytes;
        if (!A_MN) {
          tma_load_2d(a_dst, &tmA, &full[s], kc, m0);
        } else {
#pragma unroll
          for (int j = 0; j < kBM / 64; ++j)
            if (m0 + 64 * j < p.M) tma_load_2d(a_dst + j * kMNBoxBytes, &tmA, &full[s], m0 + 64 * j, kc);
        }
        if (!B_MN) {
          tma_load_2d(b_dst, &tmB, &full[s], kc, n0);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            if (n0 + 64 * j < p.N) tma_load_2d(b_dst + j * kMNBoxBytes, &tmB, &full[s], n0 + 64 * j, kc);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&full[s], ph)) {
          report_error(p.status, kTimeoutTmaFull, 2);
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kABytes);
        const uint32_t b_base = smem_u32(sB + s * C::kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ad = A_MN ? umma_desc_sw128(a_base + kk * 2048, kMNBoxBytes, 1024)
                                   : umma_desc_sw128(a_base + kk * 32, 16, 1024);
          const uint64_t bd = B_MN ? umma_desc_sw128(b_base + kk * 2048, kMNBoxBytes, 1024)
                                   : umma_desc_sw128(b_base + kk * 32, 16, 1024);
          mma_bf16_ss(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(accum);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Warp w may only read TMEM lanes [32 * (w % 4), +32): its quadrant q owns output rows m0 + 32q .. +31, one row
    // per lane. The two warps of a quadrant take alternate column chunks. The pipeline buffers are idle once the
    // accumulator is complete, so each warp stages its chunks there to make global loads/stores row-contiguous.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    const int row_base = m0 + q * 32;
    const int row = row_base + lane;
    const bool row_ok = row < p.M;
    uint32_t* stage_aux = reinterpret_cast<uint32_t*>(smem) + ew * 2 * kStageWords;
    uint32_t* stage_out = stage_aux + kStageWords;
    uint32_t ok = 1;
    if (lane == 0) ok = mbar_wait(accum, 0) ? 1u : 0u;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok && lane == 0) report_error(p.status, kTimeoutAccum, 3);
    tc_fence_after();
    constexpr int CW = BN >= 64 ? 64 : 32;  // columns per chunk (64 bf16 = one 128-byte line per row)
    constexpr int WPR = CW / 2;             // 32-bit words per row of a bf16 chunk
    constexpr int LPR = WPR / 4;            // lanes per row for 16-byte accesses
    constexpr int RPP = 32 / LPR;           // rows per pass
    if (ok && nkb > 0) {
#pragma unroll 1
      for (int c = half * CW; c < BN; c += 2 * CW) {
        const int nb = n0 + c;
        if (nb >= p.N) break;
        const int valid = min(CW, p.N - nb);
        const bool full_cols = valid == CW;
        if constexpr (EPI == kEpiDgradElu) {
          // coalesced load of the aux (ELU output) chunk, RPP rows per pass
          const __nv_bfloat16* aux = static_cast<const __nv_bfloat16*>(p.aux);
          const int lr = lane / LPR, lw = (lane % LPR) * 4;
          const bool vec = full_cols && (p.ld_aux % 8) == 0;
#pragma unroll
          for (int r0 = 0; r0 < 32; r0 += RPP) {
            const int r = r0 + lr;
            const int gr = row_base + r;
            uint32_t w4[4] = {0u, 0u, 0u, 0u};
            if (gr < p.M) {
              const __nv_bfloat16* src = aux + static_cast<size_t>(gr) * p.ld_aux + nb + 2 * lw;
              if (vec) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
                w4[0] = raw.x;
                w4[1] = raw.y;
                w4[2] = raw.z;
                w4[3] = raw.w;
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int col = 2 * (lw + i);
                  const float lo = col < valid ? __bfloat162float(src[2 * i]) : 0.f;
                  const float hi = col + 1 < valid ? __bfloat162float(src[2 * i + 1]) : 0.f;
                  w4[i] = pack_bf16x2(lo, hi);
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) stage_aux[r * 33 + lw + i] = w4[i];
          }
          __syncwarp();
        }
#pragma unroll
        for (int sub = 0; sub < CW; sub += 32) {
          float v[32];
          tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c + sub), v);
          tmem_wait_ld();
          const int sb = nb + sub;
          if constexpr (EPI == kEpiF32 || EPI == kEpiBiasEluBf16 || EPI == kEpiBiasBf16) {
            if (p.bias != nullptr) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += (sb + j < p.N) ? __ldg(p.bias + sb + j) : 0.f;
            }
          }
          if constexpr (EPI == kEpiBiasEluBf16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.f ? v[j] : __expf(v[j]) - 1.0f;
          }
          if constexpr (EPI == kEpiDgradElu) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint32_t w = stage_aux[lane * 33 + (sub + j) / 2];
              __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w);
              v[j] *= elu_grad_from_out(__low2float(h2));
              v[j + 1] *= elu_grad_from_out(__high2float(h2));
            }
            if (!row_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
          }
          if constexpr (EPI == kEpiF32 || EPI == kEpiPartialF32) {
            float* o = static_cast<float*>(p.out) + (EPI == kEpiPartialF32 ? blockIdx.z * p.split_stride : 0ll) +
                       static_cast<size_t>(row) * p.ldo + sb;
            if (row_ok) {
              if (sb + 32 <= p.N && (p.ldo % 4) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (sb + j < p.N) o[j] = v[j];
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; j += 2) stage_out[lane * 33 + (sub + j) / 2] = pack_bf16x2(v[j], v[j + 1]);
          }
          if constexpr (EPI == kEpiDgradElu) {
            if (p.colsum != nullptr) {
              // per-column sums; columns at or past N are never written out
              const float s = warp_transpose_reduce32(v);
              colsum_s[q * BN + c + sub + lane] = s;
            }
          }
        }
        if constexpr (EPI == kEpiBiasEluBf16 || EPI == kEpiBiasBf16 || EPI == kEpiDgradElu) {
          __syncwarp();
          __nv_bfloat16* outp = static_cast<__nv_bfloat16*>(p.out);
          const int lr = lane / LPR, lw = (lane % LPR) * 4;
          const bool vec = full_cols && (p.ldo % 8) == 0;
#pragma unroll
          for (int r0 = 0; r0 < 32; r0 += RPP) {
            const int r = r0 + lr;
            const int gr = row_base + r;
            if (gr < p.M) {
              __nv_bfloat16* dst = outp + static_cast<size_t>(gr) * p.ldo + nb + 2 * lw;
              const uint32_t* src = stage_out + r * 33 + lw;
              if (vec) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(src[0], src[1], src[2], src[3]);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int col = 2 * (lw + i);
                  __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&src[i]);
                  if (col < valid) dst[2 * i] = __low2bfloat16(h2);
                  if (col + 1 < valid) dst[2 * i + 1] = __high2bfloat16(h2);
                }
              }
            }
          }
          __syncwarp();
        }
      }
    }
    if constexpr (EPI == kEpiDgradElu) {
      if (p.colsum != nullptr) {
        named_barrier_sync(1, kEpiWarps * 32);
        const int t = threadIdx.x - 64;
        for (int n = t; n < BN; n += kEpiWarps * 32) {
          if (n0 + n < p.N) {
            const float s = colsum_s[n] + colsum_s[BN + n] + colsum_s[2 * BN + n] + colsum_s[3 * BN + n];
            p.colsum[static_cast<size_t>(blockIdx.x) * p.N + n0 + n] = s;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map: dims {inner, outer}, row pitch ld elements, box {box_inner, box_outer}, 128B swizzle.
bool make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
              uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
cudaError_t launch_t(const GemmParams& p, cudaStream_t stream) {
  using C = Cfg<BN, EPI>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  CUtensorMap ta, tb;
  bool ok = A_MN ? make_map(&ta, p.a, p.M, p.K, p.lda, 64, 64) : make_map(&ta, p.a, p.K, p.M, p.lda, 64, kBM);
  ok = ok && (B_MN ? make_map(&tb, p.b, p.N, p.K, p.ldb, 64, 64) : make_map(&tb, p.b, p.K, p.N, p.ldb, 64, BN));
  if (!ok) return cudaErrorInvalidValue;
  const int num_kb = (p.K + kBK - 1) / kBK;
  dim3 grid((p.M + kBM - 1) / kBM, (p.N + BN - 1) / BN, p.splits);
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(ta, tb, p, num_kb);
  return cudaGetLastError();
}

template <bool A_MN, bool B_MN, int EPI>
cudaError_t launch_bn(const GemmParams& p, cudaStream_t stream) {
  if (!B_MN && p.N <= 32) return launch_t<32, A_MN, B_MN, EPI>(p, stream);
  if (p.N <= 64) return launch_t<64, A_MN, B_MN, EPI>(p, stream);
  if (p.N <= 128) return launch_t<128, A_MN, B_MN, EPI>(p, stream);
  return launch_t<256, A_MN, B_MN, EPI>(p, stream);
}

}  // namespace

cudaError_t gemm_launch(const GemmParams& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.splits < 1) return cudaErrorInvalidValue;
  if ((p.lda % 8) != 0 || (p.ldb % 8) != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(p.a) & 15) || (reinterpret_cast<uintptr_t>(p.b) & 15)) return cudaErrorInvalidValue;
  const int num_kb = (p.K + kBK - 1) / kBK;
  if (p.splits > num_kb) return cudaErrorInvalidValue;
  if (p.splits > 1 && p.epilogue != kEpiPartialF32) return cudaErrorInvalidValue;
  if (p.epilogue == kEpiDgradElu && p.aux == nullptr) return cudaErrorInvalidValue;
  const bool am = p.a_mn_major, bm = p.b_mn_major;
  switch (p.epilogue) {
    case kEpiF32:
      if (!am && !bm) return launch_bn<false, false, kEpiF32>(p, stream);
      if (!am && bm) return launch_bn<false, true, kEpiF32>(p, stream);
      break;
    case kEpiBiasEluBf16:
      if (!am && !bm) return launch_bn<false, false, kEpiBiasEluBf16>(p, stream);
      break;
    case kEpiBiasBf16:
      if (!am && !bm) return launch_bn<false, false, kEpiBiasBf16>(p, stream);
      break;
    case kEpiDgradElu:
      if (!am && bm) return launch_bn<false, true, kEpiDgradElu>(p, stream);
      break;
    case kEpiPartialF32:
      if (am && bm) return launch_bn<true, true, kEpiPartialF32>(p, stream);
      if (!am && !bm) return launch_bn<false, false, kEpiPartialF32>(p, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace rlb
