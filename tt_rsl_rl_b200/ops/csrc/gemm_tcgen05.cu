// tcgen05 GEMM for sm_100a: TMA -> shared memory (128-byte swizzle) -> tcgen05.mma (fp32 accumulators in TMEM)
// -> tcgen05.ld epilogue with the MLP's fused elementwise work.
//
// Persistent kernel, one CTA per SM, static round-robin tile schedule (N tiles fastest, then M tiles, then split-K
// slices). TMEM holds two 128 x BN fp32 accumulators so the epilogue of tile j overlaps the MMAs of tile j + 1, and
// the TMA producer streams operand tiles through a ring of shared-memory stages across tile boundaries.
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..9  : epilogue; warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32) = output rows of its quadrant, the two
//                 warps of a quadrant splitting the column chunks
// Barriers: full/empty per ring stage (TMA <-> MMA), acc_full/acc_empty per accumulator (MMA <-> epilogue). Every
// wait is bounded (%globaltimer); a timeout records the site in the status word and the kernel unwinds.
// bf16-output epilogues work in 32-row x 32-column steps through two 2 KB buffers per warp (64-byte swizzle, so the
// row-per-thread 16-byte shared accesses are conflict-free): the data-gradient epilogue TMA-loads the next step's
// ELU-output tile while it computes the current one, and every step leaves through a TMA store.
// Every CTA fetches its own tiles from this GPU's memory; no tile load is shared between CTAs.
//
// The MLP layers of rsl_rl (rsl_rl/modules/mlp.py:91-95, Linear+ELU stacks) map onto three uses:
//   forward : H_l   = elu(H_{l-1} W_l^T + b_l)      A = H_{l-1} (K-major), B = W_l (K-major)
//   dgrad   : dZ_l  = (dZ_{l+1} W_{l+1}) * elu'(H_l) A = dZ_{l+1} (K-major), B = W_{l+1} read MN-major
//   wgrad   : dW_l  = dZ_l^T H_{l-1}                A = dZ_l (MN-major), B = H_{l-1} (MN-major), split-K partials
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "gemm_tcgen05.cuh"
#include "sm100_primitives.cuh"

namespace rlb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle atom row
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMNBoxBytes = 64 * kBK * 2;  // one {64 MN x 64 K} box
constexpr int kEpiBufBytes = 32 * 32 * 2;  // one epilogue step: 32 rows x 32 bf16 columns (64-byte rows)
constexpr int kSmemLimit = 227 * 1024;
// Recurrent-cell epilogue: per warp, five [32 rows x 16 units] fp32 blocks with a row stride of 20 floats (80 bytes:
// row-per-thread float4 accesses hit distinct banks) through which it turns row-per-thread data into row-contiguous
// 64-byte global accesses
constexpr int kRnnRowStride = 20;
constexpr int kRnnBlockFloats = 32 * kRnnRowStride;
constexpr int kRnnWarpBytes = 5 * kRnnBlockFloats * 4;
// fp32-output epilogues: per warp one [32 rows x 32 columns] block, row stride 36 floats (conflict-free float4 row
// writes and 32-lane reads); rows leave as 128-byte row-contiguous stores
constexpr int kF32RowStride = 36;
constexpr int kF32WarpBytes = 32 * kF32RowStride * 4;

// Resident CTAs per SM: the bf16-output epilogues (forward activations, data gradients that also stream the ELU
// activations in) run two CTAs per SM (BN <= 128, TMEM 2 x 2 x 128 columns) to keep 16 epilogue warps per SM; the
// fp32-output epilogues run one CTA with BN up to 256.
template <int EPI>
struct CtasPerSm {
  static constexpr int value = (EPI == kEpiDgradElu || EPI == kEpiBiasEluBf16 || EPI == kEpiBiasBf16) ? 2 : 1;
};

// WIDE: one CTA per SM with 16 epilogue warps (four per TMEM lane quadrant) and the whole shared memory for a deeper
// operand ring; otherwise CtasPerSm CTAs with 8 epilogue warps each.
template <int EPI, bool WIDE>
struct Shape {
  static constexpr int kMinBlocks = WIDE ? 1 : CtasPerSm<EPI>::value;
  static constexpr int kEpiWarps = WIDE ? 16 : 8;
  static constexpr int kThreads = 64 + kEpiWarps * 32;
};

template <int BN, int EPI, bool WIDE>
struct Cfg {
  static constexpr int kMinBlocks = Shape<EPI, WIDE>::kMinBlocks;
  static constexpr int kEpiWarps = Shape<EPI, WIDE>::kEpiWarps;
  static constexpr int kSmemBudget = kMinBlocks == 1 ? kSmemLimit : (228 * 1024) / 2 - 1024;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr bool kStaged = !(EPI == kEpiF32 || EPI == kEpiPartialF32 || EPI == kEpiRnnCell);  // bf16 via smem
  static constexpr int kStagingBytes = kStaged                 ? kEpiWarps * 2 * kEpiBufBytes
                                       : EPI == kEpiRnnCell     ? kEpiWarps * kRnnWarpBytes
                                                                : kEpiWarps * kF32WarpBytes;
  static constexpr int kBiasBytes = kStaged ? kEpiWarps * 32 * 4 : 0;
  static constexpr int kColsumBytes = EPI == kEpiDgradElu ? 2 * 4 * BN * 4 : 0;  // double-buffered by tile parity
  static constexpr int kColAccBytes = EPI == kEpiDgradElu ? kColsumMaxN * 4 : 0;   // the CTA's running column sums
  static constexpr int kBarrierBytes = 512;
  static constexpr int kFixed = 1024 /*alignment slack*/ + kStagingBytes + kBiasBytes + kColsumBytes + kColAccBytes +
                                kBarrierBytes;
  static constexpr int kStagesFit = (kSmemBudget - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  // two accumulators; the allocation is a power of two columns (192-column cell tiles allocate 512)
  static constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128 : 2 * kAccCols <= 256 ? 256 : 512;
  static constexpr int kSmemBytes = kFixed + kStages * kStageBytes;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kTmemCols * kMinBlocks <= 512, "TMEM holds 512 columns per SM");
};

struct TileCoord {
  int m0, n0, m_tile, split, kb_begin, kb_end;
};

__device__ __forceinline__ TileCoord decode_tile(int t, int n_tiles, int m_tiles, int splits, int num_kb, int BN) {
  TileCoord c;
  const int n_tile = t % n_tiles;
  const int rest = t / n_tiles;
  c.m_tile = rest % m_tiles;
  c.split = rest / m_tiles;
  c.m0 = c.m_tile * kBM;
  c.n0 = n_tile * BN;
  c.kb_begin = static_cast<int>((static_cast<long long>(c.split) * num_kb) / splits);
  c.kb_end = static_cast<int>((static_cast<long long>(c.split + 1) * num_kb) / splits);
  return c;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool WIDE>
__global__ void __launch_bounds__(Shape<EPI, WIDE>::kThreads, Shape<EPI, WIDE>::kMinBlocks)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmX,
                   const GemmParams p, int num_kb, int n_tiles, int m_tiles, int splits) {
  using C = Cfg<BN, EPI, WIDE>;
  constexpr int S = C::kStages;
  constexpr int kEpiWarps = C::kEpiWarps;
  constexpr int kPerQuad = kEpiWarps / 4;  // epilogue warps sharing a TMEM lane quadrant
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kABytes;
  uint8_t* staging = sB + S * C::kBBytes;  // 1024-byte aligned: stage sizes are multiples of 1 KB
  float* bias_smem = reinterpret_cast<float*>(staging + C::kStagingBytes);
  float* colsum_s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bias_smem) + C::kBiasBytes);
  float* colacc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(colsum_s) + C::kColsumBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(colacc) + C::kColAccBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* aux_bar = acc_empty + 2;  // two per epilogue warp (data-gradient epilogue)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + 2 * kEpiWarps);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = n_tiles * m_tiles * splits;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    for (int b = 0; b < 2 * kEpiWarps; ++b) mbar_init(&aux_bar[b], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (C::kStaged) tma_prefetch_desc(&tmO);
    if constexpr (EPI == kEpiDgradElu) tma_prefetch_desc(&tmX);
  }
  // Launched with programmatic stream serialization: the barrier setup above overlaps the previous kernel's tail.
  // Nothing before this wait touches global memory or TMEM.
  griddep_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Every CTA of this grid holds its TMEM now, so the next kernel may be scheduled: it waits for this grid's
  // completion before it allocates TMEM or touches memory, so a waiting CTA never holds what this grid needs.
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(t, n_tiles, m_tiles, splits, num_kb, BN);
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            report_error(p.status, kTimeoutSmemEmpty, 1);
            ok = false;
            break;
          }
          const int kc = kb * kBK;
          uint32_t bytes = 0;
          if (!A_MN) {
            bytes += kABytes;
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              if (tc.m0 + 64 * j < p.M) bytes += kMNBoxBytes;
          }
          if (!B_MN) {
            bytes += C::kBBytes;
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              if (tc.n0 + 64 * j < p.N) bytes += kMNBoxBytes;
          }
          mbar_arrive_expect_tx(&full[s], bytes);
          uint8_t* a_dst = sA + s * kABytes;
          uint8_t* b_dst = sB + s * C::kBBytes;
          if (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[s], kc, tc.m0);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              if (tc.m0 + 64 * j < p.M) tma_load_2d(a_dst + j * kMNBoxBytes, &tmA, &full[s], tc.m0 + 64 * j, kc);
          }
          if constexpr (EPI == kEpiRnnCell) {
            // the tile's units of every gate: G boxes of kRnnUnits rows, stacked in the B stage
            const int u0 = (t % n_tiles) * kRnnUnits;
#pragma unroll
            for (int g = 0; g < BN / kRnnUnits; ++g)
              tma_load_2d(b_dst + g * kRnnUnits * kBK * 2, &tmB, &full[s], kc, g * p.cell.H + u0);
          } else if (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[s], kc, tc.n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              if (tc.n0 + 64 * j < p.N) tma_load_2d(b_dst + j * kMNBoxBytes, &tmB, &full[s], tc.n0 + 64 * j, kc);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      uint32_t g = 0;
      bool ok = true;
      int j = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++j) {
        const TileCoord tc = decode_tile(t, n_tiles, m_tiles, splits, num_kb, BN);
        const int b = j & 1;
        const uint32_t use = static_cast<uint32_t>(j >> 1);
        if (!mbar_wait(&acc_empty[b], (use & 1) ^ 1)) {
          report_error(p.status, kTimeoutAccum, 4);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * C::kAccCols);
        for (int kb = tc.kb_begin; kb < tc.kb_end; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&full[s], ph)) {
            report_error(p.status, kTimeoutTmaFull, 2);
            ok = false;
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
            mma_bf16_ss(d, ad, bd, idesc, (kb > tc.kb_begin || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[b]);
      }
    }
  } else if constexpr (C::kStaged) {
    // ---------------- bf16-output epilogue (warps 2..9), 32 x 32 steps through two swizzled buffers -------------
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant: hardware rule warp % 4
    const int slot = ew >> 2;  // this warp takes the quadrant's 32-column steps slot, slot + kPerQuad, ...
    uint8_t* ebuf = staging + ew * 2 * kEpiBufBytes;
    float* bias_s = bias_smem + ew * 32;
    uint64_t* xbar = aux_bar + 2 * ew;
    // 64-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3); each thread owns row `lane`
    const int swz = (lane >> 1) & 3;
    // next (tile, 32-column step) of this warp whose aux tile is still to be loaded (data-gradient epilogue)
    int pt = blockIdx.x, psc = slot;
    int issued = 0, consumed = 0;
    auto seek = [&](int& t, int& sc) {
      while (t < num_tiles) {
        const int n0 = (t % n_tiles) * BN;
        if (sc * 32 < BN && n0 + sc * 32 < p.N) return;
        t += gridDim.x;
        sc = slot;
      }
    };
    auto issue_aux = [&]() {  // lane 0 only
      if (pt >= num_tiles) return;
      const TileCoord pc = decode_tile(pt, n_tiles, m_tiles, splits, num_kb, BN);
      uint8_t* dst = ebuf + (issued & 1) * kEpiBufBytes;
      bulk_wait_group_read<0>();  // the store that last read this buffer is done with it
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&xbar[issued & 1], kEpiBufBytes);
      tma_load_2d(dst, &tmX, &xbar[issued & 1], pc.n0 + psc * 32, pc.m0 + q * 32);
      ++issued;
      psc += kPerQuad;
      seek(pt, psc);
    };
    if constexpr (EPI == kEpiDgradElu) {
      seek(pt, psc);
      if (lane == 0) issue_aux();
      // the CTA's running column sums start at zero (made visible by the first tile's named barrier)
      if (p.colsum != nullptr)
        for (int n = threadIdx.x - 64; n < p.N; n += kEpiWarps * 32) colacc[n] = 0.f;
    }
    // After a timeout the warp keeps walking the tile schedule without waiting or computing, so every epilogue warp
    // still reaches each tile's column-sum barrier (a named barrier cannot time out) and the kernel unwinds.
    bool failed = false;
    int j = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++j) {
      const TileCoord tc = decode_tile(t, n_tiles, m_tiles, splits, num_kb, BN);
      const int b = j & 1;
      const uint32_t use = static_cast<uint32_t>(j >> 1);
      if (!failed) {
        uint32_t ok = 1;
        if (lane == 0) ok = mbar_wait(&acc_full[b], use & 1) ? 1u : 0u;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) report_error(p.status, kTimeoutAccum, 3);
          failed = true;
        }
      }
      tc_fence_after();
      const int row_base = tc.m0 + q * 32;
      const bool row_ok = row_base + lane < p.M;
      const uint32_t acc = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * C::kAccCols);
      float* cs = colsum_s + b * 4 * BN;
#pragma unroll 1
      for (int sc = slot; !failed && sc * 32 < BN && tc.n0 + sc * 32 < p.N; sc += kPerQuad, ++consumed) {
        const int sb = tc.n0 + sc * 32;
        uint8_t* buf = ebuf + (consumed & 1) * kEpiBufBytes;
        float v[32];
        tmem_ld_32x32b_x32(acc + static_cast<uint32_t>(sc * 32), v);
        if constexpr (EPI == kEpiDgradElu) {
          if (lane == 0) issue_aux();  // next step's ELU-output tile, one step ahead
        } else {
          if (lane == 0) bulk_wait_group_read<1>();  // the store issued two steps ago has read this buffer
          bias_s[lane] = (p.bias != nullptr && sb + lane < p.N) ? __ldg(p.bias + sb + lane) : 0.f;
        }
        __syncwarp();
        tmem_wait_ld();
        uint4* rowp = reinterpret_cast<uint4*>(buf + lane * 64);
        if constexpr (EPI == kEpiDgradElu) {
          uint32_t ok2 = mbar_wait(&xbar[consumed & 1], (consumed >> 1) & 1) ? 1u : 0u;
          if (!__all_sync(0xffffffffu, ok2)) {
            if (lane == 0) report_error(p.status, kTimeoutTmaFull, 5);
            failed = true;
            ++consumed;  // this step's aux tile is accounted for (drained below if it lands late)
            break;
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 w = rowp[c ^ swz];
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&ws[i]);
              v[8 * c + 2 * i] *= elu_grad_from_out(__low2float(h2));
              v[8 * c + 2 * i + 1] *= elu_grad_from_out(__high2float(h2));
            }
          }
          if (!row_ok) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = 0.f;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 bb = reinterpret_cast<const float4*>(bias_s)[c];  // broadcast read
            v[4 * c] += bb.x;
            v[4 * c + 1] += bb.y;
            v[4 * c + 2] += bb.z;
            v[4 * c + 3] += bb.w;
          }
          if constexpr (EPI == kEpiBiasEluBf16) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = v[jj] > 0.f ? v[jj] : __expf(v[jj]) - 1.0f;
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          rowp[c ^ swz] = make_uint4(pack_bf16x2(v[8 * c], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                                     pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
        if constexpr (EPI == kEpiDgradElu) {
          if (p.colsum != nullptr) {
            const float sum = warp_transpose_reduce32(v);  // per-column sums over this warp's 32 rows
            cs[q * BN + sc * 32 + lane] = sum;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row_base < p.M) tma_store_2d(&tmO, buf, sb, row_base);
          bulk_commit_group();
        }
      }
      // accumulator b fully read by this warp: hand it back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && !failed) mbar_arrive(&acc_empty[b]);
      if constexpr (EPI == kEpiDgradElu) {
        if (p.colsum != nullptr) {
          named_barrier_sync(1, kEpiWarps * 32);
          const int tt = threadIdx.x - 64;
          for (int n = tt; n < BN; n += kEpiWarps * 32) {
            if (tc.n0 + n < p.N) colacc[tc.n0 + n] += (cs[n] + cs[BN + n]) + (cs[2 * BN + n] + cs[3 * BN + n]);
          }
        }
      }
    }
    if constexpr (EPI == kEpiDgradElu) {
      // one partial row per CTA (tiles of this CTA summed in schedule order); rows of CTAs that this launch does not
      // have are cleared by CTA 0, so the reduction over all colsum_rows rows never sums stale values
      if (p.colsum != nullptr) {
        named_barrier_sync(1, kEpiWarps * 32);
        const int tt = threadIdx.x - 64;
        for (int n = tt; n < p.N; n += kEpiWarps * 32) {
          p.colsum[static_cast<size_t>(blockIdx.x) * p.N + n] = colacc[n];
          if (blockIdx.x == 0)
            for (int r = gridDim.x; r < p.colsum_rows; ++r) p.colsum[static_cast<size_t>(r) * p.N + n] = 0.f;
        }
      }
    }
    if (lane == 0) {
      // aux tiles still in flight after an early exit land before the CTA's shared memory is released; a tile whose
      // wait already timed out is waited for once more (bounded)
      const int first = failed ? consumed - 1 : consumed;
      for (int k = first < 0 ? 0 : first; k < issued; ++k) mbar_wait(&xbar[k & 1], (k >> 1) & 1);
      bulk_wait_group<0>();  // outputs written before the kernel ends
    }
    __syncwarp();
  } else if constexpr (EPI == kEpiRnnCell) {
    // ---------------- recurrent-cell epilogue (warps 2..9) ----------------
    // A thread owns one row (TMEM lane); the kPerQuad warps of a quadrant split the tile's kRnnUnits units in chunks
    // of 32. Per chunk: the G gate columns of the accumulator, + b_hh, then the cell four units at a time with
    // 16-byte loads of gi / the input state and 16-byte (fp32) or 8-byte (bf16) stores of every output.
    constexpr int G = BN / kRnnUnits;
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant: hardware rule warp % 4
    const int slot = ew >> 2;
    const RnnCellEpi& e = p.cell;
    const int H = e.H;
    int j = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++j) {
      const TileCoord tc = decode_tile(t, n_tiles, m_tiles, splits, num_kb, BN);
      const int u0 = (t % n_tiles) * kRnnUnits;
      const int b = j & 1;
      const uint32_t use = static_cast<uint32_t>(j >> 1);
      uint32_t ok = 1;
      if (lane == 0) ok = mbar_wait(&acc_full[b], use & 1) ? 1u : 0u;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) report_error(p.status, kTimeoutAccum, 6);
        break;
      }
      tc_fence_after();
      const long long row = tc.m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t acc = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * C::kAccCols);
      const float keep = (row_ok && e.done) ? 1.0f - __ldg(e.done + row) : 1.0f;
      // Global memory is accessed row-contiguously: lane l moves 16 bytes of row (l >> 2) + 8 i, i = 0..3 (four
      // lanes per 64-byte row segment); the warp's shared blocks turn that into one row per thread and back.
      const long long row_base = tc.m0 + q * 32;
      const int cr = lane >> 2, cq = lane & 3;
      float* const wbuf = reinterpret_cast<float*>(staging) + ew * (kRnnWarpBytes / 4);
      // copies between global rows [row_base, row_base + 32) x 16 columns and block `blk` of the warp's buffer
      auto gather = [&](const float* src, long long ld, int blk) {
        float4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const long long r = row_base + cr + 8 * i;
          v[i] = r < p.M ? __ldg(reinterpret_cast<const float4*>(src + r * ld) + cq) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<float4*>(wbuf + blk * kRnnBlockFloats + (cr + 8 * i) * kRnnRowStride + 4 * cq) = v[i];
      };
      auto scatter = [&](float* dst, long long ld, int blk) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const long long r = row_base + cr + 8 * i;
          const float4 v =
              *reinterpret_cast<const float4*>(wbuf + blk * kRnnBlockFloats + (cr + 8 * i) * kRnnRowStride + 4 * cq);
          if (r < p.M) *(reinterpret_cast<float4*>(dst + r * ld) + cq) = v;
        }
      };
      auto put_row = [&](int blk, const float (&v)[16]) {  // this thread's row of a block
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<float4*>(wbuf + blk * kRnnBlockFloats + lane * kRnnRowStride + 4 * q4) =
              make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
      };
      auto get_row = [&](int blk, float (&v)[16]) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 t4 = *reinterpret_cast<const float4*>(wbuf + blk * kRnnBlockFloats + lane * kRnnRowStride + 4 * q4);
          v[4 * q4] = t4.x;
          v[4 * q4 + 1] = t4.y;
          v[4 * q4 + 2] = t4.z;
          v[4 * q4 + 3] = t4.w;
        }
      };
      // bf16 rows (32 bytes) of block `blk`: thread-row packs, then lane l stores 16 bytes of row (l >> 1) + 16 i
      auto scatter_bf16 = [&](void* dst, long long ld, int blk, const float (&v)[16], float scale) {
        uint4* rowp = reinterpret_cast<uint4*>(wbuf + blk * kRnnBlockFloats + lane * 12);  // 48-byte rows
        rowp[0] = make_uint4(pack_bf16x2(v[0] * scale, v[1] * scale), pack_bf16x2(v[2] * scale, v[3] * scale),
                             pack_bf16x2(v[4] * scale, v[5] * scale), pack_bf16x2(v[6] * scale, v[7] * scale));
        rowp[1] = make_uint4(pack_bf16x2(v[8] * scale, v[9] * scale), pack_bf16x2(v[10] * scale, v[11] * scale),
                             pack_bf16x2(v[12] * scale, v[13] * scale), pack_bf16x2(v[14] * scale, v[15] * scale));
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int rr = (lane >> 1) + 16 * i;
          const long long r = row_base + rr;
          const uint4 w = reinterpret_cast<const uint4*>(wbuf + blk * kRnnBlockFloats + rr * 12)[lane & 1];
          if (r < p.M)
            reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst) + r * ld + (lane & 1) * 8)[0] = w;
        }
      };
#pragma unroll 1
      for (int c = slot * 16; c < kRnnUnits; c += kPerQuad * 16) {
        const int u = u0 + c;  // first hidden unit of the sub-chunk
        float gh[G][16];
#pragma unroll
        for (int g = 0; g < G; ++g) tmem_ld_32x32b_x16(acc + static_cast<uint32_t>(g * kRnnUnits + c), gh[g]);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float bl = __ldg(p.bias + g * H + u + (lane & 15));  // lanes l and l + 16 hold the bias of unit u + l
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) gh[g][jj] += __shfl_sync(0xffffffffu, bl, jj);
        }
        // inputs: the G gate blocks of gi and the state block (h_in for GRU, c_in for LSTM)
#pragma unroll
        for (int g = 0; g < G; ++g) gather(e.gi + g * H + u, e.ld_gi, g);
        if constexpr (G == 4) gather(e.c_in + u, e.ld_c_in, G);
        else gather(e.h_in + u, e.ld_h_in, G);
        __syncwarp();
        float x[G][16], st[16];
#pragma unroll
        for (int g = 0; g < G; ++g) get_row(g, x[g]);
        get_row(G, st);
        __syncwarp();
        // the cell; saved activations go straight to this thread's row of blocks 0 .. S-1 (inputs are in registers)
        constexpr int S = G == 4 ? 5 : 4;
        float hn[16], cn[16];
        float* my = wbuf + lane * kRnnRowStride;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          if constexpr (G == 3) {  // GRU: r, z, n; st = h_in
            const float r = 1.0f / (1.0f + __expf(-(x[0][k] + gh[0][k])));
            const float z = 1.0f / (1.0f + __expf(-(x[1][k] + gh[1][k])));
            const float ghn = gh[2][k];
            const float n = tanhf(x[2][k] + r * ghn);
            hn[k] = (1.0f - z) * n + z * st[k];
            cn[k] = 0.f;
            my[k] = r;
            my[kRnnBlockFloats + k] = z;
            my[2 * kRnnBlockFloats + k] = n;
            my[3 * kRnnBlockFloats + k] = ghn;
          } else {  // LSTM: i, f, g, o; st = c_in
            const float ig = 1.0f / (1.0f + __expf(-(x[0][k] + gh[0][k])));
            const float fg = 1.0f / (1.0f + __expf(-(x[1][k] + gh[1][k])));
            const float gg = tanhf(x[2][k] + gh[2][k]);
            const float og = 1.0f / (1.0f + __expf(-(x[3][k] + gh[3][k])));
            cn[k] = fg * st[k] + ig * gg;
            const float tcn = tanhf(cn[k]);
            hn[k] = og * tcn;
            my[k] = ig;
            my[kRnnBlockFloats + k] = fg;
            my[2 * kRnnBlockFloats + k] = gg;
            my[3 * kRnnBlockFloats + k] = og;
            my[4 * kRnnBlockFloats + k] = tcn;
          }
        }
        __syncwarp();
        if (e.save) {
#pragma unroll
          for (int sidx = 0; sidx < S; ++sidx) scatter(e.save + sidx * H + u, e.ld_save, sidx);
        }
        __syncwarp();
        // fp32 states: h', h' (1 - done), c', c' (1 - done)
        float hk[16], ck[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          hk[k] = hn[k] * keep;
          ck[k] = cn[k] * keep;
        }
        put_row(0, hn);
        put_row(1, hk);
        if constexpr (G == 4) {
          put_row(2, cn);
          put_row(3, ck);
        }
        __syncwarp();
        if (e.h_out) scatter(e.h_out + u, e.ld_h_out, 0);
        if (e.next_h) scatter(e.next_h + u, e.ld_next_h, 1);
        if constexpr (G == 4) {
          if (e.c_out) scatter(e.c_out + u, e.ld_c_out, 2);
          if (e.next_c) scatter(e.next_c + u, e.ld_next_c, 3);
        }
        __syncwarp();
        if (e.h_out_bf16) scatter_bf16(static_cast<__nv_bfloat16*>(e.h_out_bf16) + u, e.ld_h_out_bf16, 0, hn, 1.0f);
        if (e.next_h_bf16)
          scatter_bf16(static_cast<__nv_bfloat16*>(e.next_h_bf16) + u, e.ld_next_h_bf16, 1, hn, keep);
        __syncwarp();
      }
      // accumulator b fully read by this warp: hand it back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  } else {
    // ---------------- fp32-output epilogue (warps 2..9) ----------------
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant: hardware rule warp % 4
    const int slot = ew >> 2;
    constexpr int CW = BN >= 64 ? 64 : 32;  // columns per chunk
    float* const fbuf = reinterpret_cast<float*>(staging) + ew * (kF32WarpBytes / 4);
    // 16-byte row stores need 16-byte aligned rows
    const bool vec_ok = (p.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                        (EPI != kEpiPartialF32 || p.split_stride % 4 == 0);
    const int wcols = p.out_cols > p.N ? p.out_cols : p.N;  // writable columns of a row
    int j = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++j) {
      const TileCoord tc = decode_tile(t, n_tiles, m_tiles, splits, num_kb, BN);
      const int b = j & 1;
      const uint32_t use = static_cast<uint32_t>(j >> 1);
      uint32_t ok = 1;
      if (lane == 0) ok = mbar_wait(&acc_full[b], use & 1) ? 1u : 0u;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) report_error(p.status, kTimeoutAccum, 3);
        break;
      }
      tc_fence_after();
      const uint32_t acc = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * C::kAccCols);
#pragma unroll 1
      for (int c = slot * CW; c < BN; c += kPerQuad * CW) {
        const int nb = tc.n0 + c;
        if (nb >= p.N) break;
#pragma unroll
        for (int sub = 0; sub < CW; sub += 32) {
          float v[32];
          tmem_ld_32x32b_x32(acc + static_cast<uint32_t>(c + sub), v);
          tmem_wait_ld();
          const int sb = nb + sub;
          if constexpr (EPI == kEpiF32) {
            if (p.bias != nullptr) {
              // lane l holds bias[sb + l]; element j takes it by shuffle
              const float my_bias = (sb + lane < p.N) ? __ldg(p.bias + sb + lane) : 0.f;
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) v[jj] += __shfl_sync(0xffffffffu, my_bias, jj);
            }
          }
          // the warp's 32 x 32 block goes through shared memory so that rows leave contiguously (a row-per-thread
          // store would touch 32 rows per instruction)
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4)
            *reinterpret_cast<float4*>(fbuf + lane * kF32RowStride + 4 * c4) =
                make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
          __syncwarp();
          float* o = static_cast<float*>(p.out) +
                     (EPI == kEpiPartialF32 ? static_cast<long long>(tc.split) * p.split_stride : 0ll) + sb;
          const long long row0 = tc.m0 + q * 32;
          if (vec_ok && sb + 32 <= wcols) {
            // lane l: 16 bytes of row 4 i + l / 8 (eight lanes per 128-byte row)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = 4 * i + (lane >> 3);
              const float4 val = *reinterpret_cast<const float4*>(fbuf + rr * kF32RowStride + 4 * (lane & 7));
              if (row0 + rr < p.M) *reinterpret_cast<float4*>(o + (row0 + rr) * p.ldo + 4 * (lane & 7)) = val;
            }
          } else {
            // lane l: column sb + l of every row
#pragma unroll 4
            for (int rr = 0; rr < 32; ++rr)
              if (row0 + rr < p.M && sb + lane < p.N) o[(row0 + rr) * p.ldo + lane] = fbuf[rr * kF32RowStride + lane];
          }
          __syncwarp();
        }
      }
      // accumulator b fully read by this warp: hand it back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
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
              uint32_t box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  });
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool WIDE>
cudaError_t launch_t(const GemmParams& p, cudaStream_t stream) {
  using C = Cfg<BN, EPI, WIDE>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI, WIDE>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  CUtensorMap ta, tb;
  bool ok = A_MN ? make_map(&ta, p.a, p.M, p.K, p.lda, 64, 64) : make_map(&ta, p.a, p.K, p.M, p.lda, 64, kBM);
  // K-major B: one box per tile, or per gate of the tile's units in the recurrent-cell epilogue
  const uint32_t b_rows = EPI == kEpiRnnCell ? static_cast<uint32_t>(kRnnUnits) : static_cast<uint32_t>(BN);
  ok = ok && (B_MN ? make_map(&tb, p.b, p.N, p.K, p.ldb, 64, 64) : make_map(&tb, p.b, p.K, p.N, p.ldb, 64, b_rows));
  // epilogue maps: bf16 output (TMA store) and ELU-output aux (TMA load), 32 x 32 boxes with 64-byte swizzle
  CUtensorMap to = ta, tx = ta;
  if constexpr (C::kStaged) ok = ok && make_map(&to, p.out, p.N, p.M, p.ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if constexpr (EPI == kEpiDgradElu)
    ok = ok && make_map(&tx, p.aux, p.N, p.M, p.ld_aux, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!ok) return cudaErrorInvalidValue;
  const int num_kb = (p.K + kBK - 1) / kBK;
  const int m_tiles = (p.M + kBM - 1) / kBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const long long tiles = static_cast<long long>(m_tiles) * n_tiles * p.splits;
  if (tiles > (1ll << 31) - 1) return cudaErrorInvalidValue;
  const long long slots = static_cast<long long>(sm_count()) * C::kMinBlocks;
  const int grid = static_cast<int>(tiles < slots ? tiles : slots);
  if (EPI == kEpiDgradElu && p.colsum != nullptr && grid > p.colsum_rows) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Shape<EPI, WIDE>::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, to, tx, p, num_kb, n_tiles, m_tiles, p.splits);
}

// Layout choice for the bf16-output epilogues. Measured on the benchmark shapes (393,216 rows): the one-CTA,
// 16-epilogue-warp layout (deeper operand ring, 256-column tiles) is faster for wide outputs (forward 96->512 and
// 512->256, data gradient 256->512: 4-12%) and slower for narrow ones (outputs of 128 or 256 columns in the data
// gradient, 128 in the forward pass: 5-20%). RLB_GEMM_WIDE=0 / 1 in the environment forces one layout (read once).
int wide_override() {
  static const int v = [] {
    const char* e = std::getenv("RLB_GEMM_WIDE");
    return e == nullptr ? -1 : (e[0] == '1' ? 1 : 0);
  }();
  return v;
}

template <int EPI>
bool use_wide(int N) {
  const int o = wide_override();
  if (o >= 0) return o == 1;
  return EPI == kEpiDgradElu ? N >= 512 : N >= 256;
}

template <bool A_MN, bool B_MN, int EPI, bool WIDE>
cudaError_t launch_bn_t(const GemmParams& p, cudaStream_t stream) {
  constexpr bool one_cta = Shape<EPI, WIDE>::kMinBlocks == 1;
  if (!B_MN && p.N <= 32) return launch_t<32, A_MN, B_MN, EPI, WIDE>(p, stream);
  if (p.N <= 64) return launch_t<64, A_MN, B_MN, EPI, WIDE>(p, stream);
  if constexpr (EPI == kEpiF32) {
    // few row tiles (a recurrent step of a few thousand rows): narrower tiles, so that at least half the SMs work
    // (a 4096 x 256 output with K = 768 runs on 128 CTAs instead of 32)
    const int m_tiles = (p.M + kBM - 1) / kBM, half = sm_count() / 2;
    if (m_tiles * ((p.N + 127) / 128) < half) return launch_t<64, A_MN, B_MN, EPI, WIDE>(p, stream);
    if (p.N > 128 && m_tiles * ((p.N + 255) / 256) < half) return launch_t<128, A_MN, B_MN, EPI, WIDE>(p, stream);
  }
  if (p.N <= 128 || !one_cta) return launch_t<128, A_MN, B_MN, EPI, WIDE>(p, stream);
  if constexpr (one_cta) return launch_t<256, A_MN, B_MN, EPI, WIDE>(p, stream);
  return cudaErrorInvalidValue;
}

template <bool A_MN, bool B_MN, int EPI>
cudaError_t launch_bn(const GemmParams& p, cudaStream_t stream) {
  constexpr bool staged = EPI == kEpiDgradElu || EPI == kEpiBiasEluBf16 || EPI == kEpiBiasBf16;
  if constexpr (staged) {
    if (use_wide<EPI>(p.N)) return launch_bn_t<A_MN, B_MN, EPI, true>(p, stream);
  }
  return launch_bn_t<A_MN, B_MN, EPI, false>(p, stream);
}

}  // namespace

// Programmatic dependent launch of the framework's kernels (the next launch's setup overlaps this one's tail);
// RLB_PDL=0 in the environment turns it off (read once).
bool pdl_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("RLB_PDL");
    return e == nullptr || e[0] != '0';
  }();
  return v;
}

cudaError_t gemm_launch(const GemmParams& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.splits < 1) return cudaErrorInvalidValue;
  if ((p.lda % 8) != 0 || (p.ldb % 8) != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(p.a) & 15) || (reinterpret_cast<uintptr_t>(p.b) & 15)) return cudaErrorInvalidValue;
  const int num_kb = (p.K + kBK - 1) / kBK;
  if (p.splits > num_kb) return cudaErrorInvalidValue;
  if (p.splits > 1 && p.epilogue != kEpiPartialF32) return cudaErrorInvalidValue;
  if (p.epilogue == kEpiDgradElu && p.aux == nullptr) return cudaErrorInvalidValue;
  if (p.out_cols != 0 && (p.epilogue != kEpiF32 || p.out_cols < p.N || p.out_cols > p.ldo)) return cudaErrorInvalidValue;
  if (p.epilogue == kEpiDgradElu && p.colsum != nullptr && (p.N > kColsumMaxN || p.colsum_rows < 1))
    return cudaErrorInvalidValue;
  const bool staged = p.epilogue == kEpiBiasEluBf16 || p.epilogue == kEpiBiasBf16 || p.epilogue == kEpiDgradElu;
  // TMA epilogue rules: 16-byte aligned bases, row pitches that are multiples of 16 bytes
  if (staged && ((p.ldo % 8) != 0 || (reinterpret_cast<uintptr_t>(p.out) & 15))) return cudaErrorInvalidValue;
  if (p.epilogue == kEpiDgradElu && ((p.ld_aux % 8) != 0 || (reinterpret_cast<uintptr_t>(p.aux) & 15)))
    return cudaErrorInvalidValue;
  const bool am = p.a_mn_major, bm = p.b_mn_major;
  if (p.epilogue == kEpiRnnCell) {
    const RnnCellEpi& e = p.cell;
    const int G = e.lstm ? 4 : 3;
    auto f32ok = [](const void* q, long long ld) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0 && ld % 4 == 0; };
    auto bf16ok = [](const void* q, long long ld) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0 && ld % 8 == 0; };
    if (am || bm || e.H <= 0 || e.H % kRnnUnits != 0 || p.K != e.H || p.N != G * e.H || p.bias == nullptr ||
        e.gi == nullptr || !f32ok(e.gi, e.ld_gi) || (e.lstm ? e.c_in == nullptr : e.h_in == nullptr))
      return cudaErrorInvalidValue;
    if ((e.h_in && !f32ok(e.h_in, e.ld_h_in)) || (e.c_in && !f32ok(e.c_in, e.ld_c_in)) ||
        (e.h_out && !f32ok(e.h_out, e.ld_h_out)) || (e.c_out && !f32ok(e.c_out, e.ld_c_out)) ||
        (e.next_h && !f32ok(e.next_h, e.ld_next_h)) || (e.next_c && !f32ok(e.next_c, e.ld_next_c)) ||
        (e.save && !f32ok(e.save, e.ld_save)) || (e.h_out_bf16 && !bf16ok(e.h_out_bf16, e.ld_h_out_bf16)) ||
        (e.next_h_bf16 && !bf16ok(e.next_h_bf16, e.ld_next_h_bf16)))
      return cudaErrorInvalidValue;
    return e.lstm ? launch_t<4 * kRnnUnits, false, false, kEpiRnnCell, false>(p, stream)
                  : launch_t<3 * kRnnUnits, false, false, kEpiRnnCell, false>(p, stream);
  }
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
