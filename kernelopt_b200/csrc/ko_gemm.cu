// fp32-grade GEMM with fused bias + activation on the B200 5th-generation tensor cores (tcgen05, kind::tf32).
//
//   out[M][N] = act(x[M][K] @ W[K][N] + bias[N])
//
// Semantics: the reference's fused fc1 kernel fast_rfdetr/kernels.py:188-266 (gemm_bias_gelu_f32, with the
// erf GELU epilogue; here the erf is Abramowitz & Stegun 7.1.26) and its unfused form model.py:142-143 (lin + 0.5*y*(1+erf(y/sqrt 2))).
//
// Precision: 3xTF32 (the error-compensated split of Ootomo & Yokota, 2022, also known as CUTLASS "3xTF32").
// Every operand is split as v = hi + lo with hi = tf32_rn(v) and lo = tf32_rn(v - hi); the tensor cores
// accumulate hi*hi + hi*lo + lo*hi in fp32 in tensor memory, which leaves an error of about 2^-21 relative per
// product — the same order as a plain fp32 dot product of this length. The weight split is done once
// (ko_pack_weight_tf32x3); the activation split happens on chip, inside the pipeline, from the fp32 tile that
// TMA brought in, so x is read from HBM exactly once.
//
// Kernel structure (persistent, one CTA per SM, 576 threads, warp-specialised):
//   warp 0      TMA producer: x tile [128 x BK] and W_hi/W_lo tiles [BN x BK] per k-block, swizzled
//   warp 1      allocates TMEM; one lane issues the tcgen05.mma (3 products per 8-wide k-step)
//   warps 2-9   split the x tile: hi in place and lo into a second buffer (same layout) in shared memory, or,
//               for 192-wide tiles, hi and lo into the stage's slot of tensor memory, where the MMA reads A
//               (the "TS" form; only B then comes from shared memory); two groups of four warps take
//               alternate k-blocks
//   warps 10-17 epilogue: TMEM -> registers (tcgen05.ld), + bias, activation, a swizzled 32x32 tile in shared
//               memory per warp, TMA store (two warps per TMEM lane quadrant)
// Two TMEM accumulators let the epilogue of tile i overlap the MMAs of tile i+1 (one, where the correction
// accumulator of SPLIT, below, leaves no room for a second).
// Two more forms share this kernel:
//   * the LayerNorm epilogue (EPI_LN): out-projection / fc2 / conv + bias, * layer scale, + residual, then a
//     LayerNorm over whole rows; rows wider than one tile are split over a cluster of two CTAs that swap
//     their row statistics through distributed shared memory;
//   * the implicit 3x3 convolution (conv_c > 0): each k-block is one tap's channel slice, loaded by TMA from
//     the image rows shifted by that tap; the split warps zero the rows whose shifted pixel is padding.
// Every wait on an mbarrier is bounded (2 s); on timeout the CTA stops, drains what it issued, frees TMEM and
// reports KO_ERR_DEVICE_TIMEOUT through dev_status.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "ko_common.cuh"

namespace {

using namespace kodev;

constexpr int BM = 128;
constexpr int kTransformWarp0 = 2;   // warps 2-9: two groups of four split alternate k-blocks
constexpr int kEpilogueWarp0 = 10;   // warps 10-17: two warps per TMEM lane quadrant
constexpr int kThreads = 18 * 32;
constexpr uint32_t kStoreTileBytes = 32 * 32 * 4;                   // one epilogue warp's 32x32 output tile
constexpr uint32_t kStoreBytes = 8 * kStoreTileBytes;               // 32 KB of staging for the TMA stores
constexpr size_t kSmemBudget = 224 * 1024 - kStoreBytes;  // stage buffers; staging, barriers, slack on top
constexpr uint32_t kBarBytes = 512;                        // mbarriers, the TMEM address and the abort flag

// BN: tile width (MMA N). BKB: bytes of K per k-block row (128 -> 128-byte swizzle, 64 -> 64-byte swizzle).
// SPLIT: accumulate the small hi*lo + lo*hi terms in their own TMEM accumulator and add it to the hi*hi
// accumulator in the epilogue. The tensor core's fp32 accumulation drops low-order bits at every MMA; with a
// single accumulator the 2 x K/8 correction MMAs land on a large running sum, which makes the error grow with
// K. With SPLIT they land on a small one, and the large sum sees only K/8 additions.
// Epilogue kinds. EPI_ACT: out = act(acc + bias). EPI_LN: v = resid + (acc + bias) * scale over whole rows
// (the N columns of a row are split over the CTAs of a cluster), y = act(LayerNorm(v) * gamma + beta).
constexpr int EPI_ACT = 0;
constexpr int EPI_LN = 1;

// Row statistics exchange of the LayerNorm epilogue: per tile parity, the two epilogue warps of a lane
// quadrant publish (mean, M2) of their half of the row [2][2][128] float2, and the cluster peer's CTA-level
// (mean, M2) lands in [2][128] float2; two mbarriers count the peer's arrivals, four (one per lane quadrant)
// the two warps of a pair, and eight or sixteen (one per epilogue warp and staging tile) the TMA loads into
// the warps' staging tiles.
constexpr uint32_t kLnStatBytes = 2 * 2 * 128 * 8 + 2 * 128 * 8 + 2 * 8 + 4 * 8 + 16 * 8;
constexpr uint32_t kLnStatRegion = 6400 + 4 * 256 * 4;  // + the CTA's column slice of bias, scale, gamma, beta
static_assert(kLnStatBytes <= kLnStatRegion, "stat region");

template <int BN, int BKB, bool SPLIT, int EPI = EPI_ACT>
struct Cfg {
  static constexpr int kBK = BKB / 4;                       // fp32 elements per k-block
  static constexpr uint32_t kATileBytes = BM * BKB;
  static constexpr uint32_t kBTileBytes = BN * BKB;
  // A from tensor memory (the split warps write x_hi / x_lo into a TMEM slot per stage, the MMA reads A there
  // and only B from shared memory) for 192-wide tiles, where the accumulators leave 128 TMEM columns free.
  static constexpr bool kTSA = BN == 192 && BKB == 64;
  static constexpr uint32_t kStageBytes = (kTSA ? 1 : 2) * kATileBytes + 2 * kBTileBytes;
  // LayerNorm epilogue without the correction accumulator: a second staging tile per epilogue warp (at kStg2Off
  // from the first set, 1024-byte aligned, after the statistics region), so a chunk's residual load overlaps the
  // previous chunk and a store's read-back does not hold up the next chunk. With the correction accumulator the
  // 32 KB would cost fc2 a pipeline stage (measured 593 -> 669 us at 64 frames), so those variants keep one tile.
  static constexpr int kStgTiles = (EPI == EPI_LN && !SPLIT) ? 2 : 1;
  static constexpr uint32_t kStg2Off = (kStoreBytes + kBarBytes + kLnStatRegion + 1023) / 1024 * 1024;
  static constexpr uint32_t kStatBytes =
      EPI == EPI_LN ? (kStgTiles == 2 ? kStg2Off - kBarBytes : kLnStatRegion) : 0;
  static constexpr int kStagesRaw = static_cast<int>((kSmemBudget - kStatBytes) / kStageBytes);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  // The A slots form their own ring of 4 (k-block kit uses slot kit % 4), so TMA can run more stages ahead
  // than there are slots.
  static constexpr int kASlots = 4;
  static constexpr uint32_t kASlotCols = 2 * kBK;                    // A_hi | A_lo of one k-block in TMEM
  static constexpr uint32_t kATmemCols = kTSA ? kASlots * kASlotCols : 0;
  static constexpr uint32_t kAccCols = BN * (SPLIT ? 2 : 1);  // TMEM columns of one tile's accumulator(s)
  static constexpr int kAccBufs = (2 * kAccCols + kATmemCols <= 512) ? 2 : 1;
  static constexpr uint32_t kAOffCol = kAccBufs * kAccCols;  // first TMEM column of the A slots
  static constexpr uint32_t kTmemNeed = kAccBufs * kAccCols + kATmemCols;
  static constexpr uint32_t kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                        : kTmemNeed <= 256 ? 256 : 512;
  static constexpr uint32_t kTxBytes = kATileBytes + 2 * kBTileBytes;
  static constexpr size_t kSmemBytes =
      1024 /*align slack*/ + kStages * kStageBytes + kStoreBytes + kBarBytes + kStatBytes;
  // Stage st's `full` barrier for k-block it is full[2 st + it % 2] (the split group of it's parity waits on it):
  // it is used every kFullPeriod k-blocks, so phase = (it / kFullPeriod) & 1.
  static constexpr uint32_t kFullPeriod = kStages % 2 == 0 ? kStages : 2 * kStages;
  static constexpr uint32_t kSbo = 8 * BKB;                 // bytes between 8-row groups
  static constexpr uint32_t kLayout = BKB == 128 ? 2u : 4u;  // descriptor layout: 128B / 64B swizzle
  static_assert(kStages >= 2, "stage does not fit");
  static_assert(kTmemNeed <= 512, "TMEM overflow");
  static_assert((4 * kStages + 10) * 8 <= kBarBytes, "barrier area");
};

struct GemmArgs {
  const float* bias;
  float* out;
  int* dev_status;
  int M, N, K, act;
  int m_tiles, n_tiles, k_blocks;
  // EPI_LN only
  const float* scale;  // per-column multiplier of (acc + bias), or null (1)
  const float* resid;  // residual added before the LayerNorm [M][N], or null
  const float* gamma;
  const float* beta;
  float eps;
  int write_v;  // store v = resid + (acc + bias) * scale through map_v
  int cs;       // CTAs per cluster = N / BN
  // Implicit 3x3 convolution (stride 1, zero padding 1) when conv_c > 0: x is an NHWC image batch
  // [M = batch * conv_h * conv_w][conv_c], K = 9 * conv_c in (ky, kx, c) order, and k-block kb reads the rows of
  // x shifted by (ky - 1) * conv_w + (kx - 1) for tap ky * 3 + kx; rows whose shifted pixel lies outside the
  // image are zeroed by the split warps.
  int conv_h, conv_w, conv_c;
  // EPI_ACT only: out = act(acc + bias + addend) with addend[row * ld_add + col] for col < add_cols (a per-element
  // term, e.g. the product of a second operand that the caller computed once for several GEMMs), or null
  const float* addend;
  int ld_add, add_cols;
};

// Tiles of one CTA. EPI_ACT: tile t of the m_tiles x n_tiles grid, CTAs strided over tiles. EPI_LN: tile t is
// row block t; the cs CTAs of a cluster take the same row block, CTA rank r the columns [r*BN, (r+1)*BN).
template <int EPI>
struct TileSched {
  int first, step, count, n_tiles, col0;
  __device__ explicit TileSched(const GemmArgs& a, int bn) {
    if (EPI == EPI_LN) {
      first = a.cs > 1 ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
      step = a.cs > 1 ? static_cast<int>(cluster_count_x()) : static_cast<int>(gridDim.x);
      count = a.m_tiles;
      n_tiles = 1;
      col0 = (a.cs > 1 ? static_cast<int>(cluster_ctarank()) : 0) * bn;
    } else {
      first = blockIdx.x;
      step = gridDim.x;
      count = a.m_tiles * a.n_tiles;
      n_tiles = a.n_tiles;
      col0 = 0;
    }
  }
  __device__ int m0(int tile) const { return (tile / n_tiles) * BM; }
  __device__ int n0(int tile, int bn) const { return (tile % n_tiles) * bn + col0; }
};

// GELU(v) = v * Phi(v), Phi the standard normal CDF = (1 + erf(v / sqrt 2)) / 2, with erfc(x) for x >= 0 from
// Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26: erfc(x) = t (a1 + t (a2 + ... + t a5))
// exp(-x^2), t = 1 / (1 + p x), absolute error below 1.5e-7. With x = |v| / sqrt 2 and q = erfc(x) / 2 (the
// factors 1/sqrt 2 and 1/2 folded into p and the a_i): Phi(v) = 1 - q for v >= 0 and q for v < 0.
__device__ __forceinline__ float gelu_as7126(float v) {
  const float ax = fabsf(v);
  const float t = __fdividef(1.0f, fmaf(0.3275911f * 0.7071067811865476f, ax, 1.0f));
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 0.5f * 1.061405429f, 0.5f * -1.453152027f),
                                               0.5f * 1.421413741f), 0.5f * -0.284496736f), 0.5f * 0.254829592f);
  float e;  // exp(-v^2 / 2) as 2^(-v^2 log2(e) / 2)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(v * v * -0.7213475204444817f));
  const float q = poly * e;
  const float vq = v * q;
  // q underflows to 0 for large |v|: GELU(v) = v there (+inf included, where v * q would be inf * 0), and
  // v * q keeps -inf -> NaN, as 0.5 * v * (1 + erf(v / sqrt 2)) gives
  return v >= 0.0f ? (q > 0.0f ? v - vq : v) : vq;
}

__device__ __forceinline__ float apply_act(float v, int act) {
#ifdef KO_GELU_ERFF  // measurement builds: CUDA's erff instead of A&S 7.1.26, to size the formula's share of error
  if (act == KO_ACT_GELU) return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
#endif
  if (act == KO_ACT_GELU) return gelu_as7126(v);
  if (act == KO_ACT_RELU) return fmaxf(v, 0.0f);
  return v;
}

// K-major operand descriptor for a swizzled tile (see smem_desc_k_sw128 for the field layout).
template <uint32_t kLayout, uint32_t kSbo>
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
         (static_cast<uint64_t>((kSbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(kLayout) << 61);
}

// TMEM store of 32 lanes x 32 consecutive columns (the inverse of tmem_ld_32x32b_x32).
__device__ __forceinline__ void tmem_store_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_store_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// (mean, M2) of two equal-sized groups of n values each, combined in the order (a, b) (Chan et al., 1979).
__device__ __forceinline__ float2 combine_stats(float2 a, float2 b, float n) {
  const float d = b.x - a.x;
  return make_float2(a.x + 0.5f * d, a.y + b.y + d * d * (0.5f * n));
}

__device__ __forceinline__ float ln_act(float r, int act) {
  return act == KO_ACT_SILU ? r / (1.0f + expf(-r)) : r;
}

template <int BN, int BKB, bool SPLIT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_whi,
                       const __grid_constant__ CUtensorMap map_wlo, const __grid_constant__ CUtensorMap map_out,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_r,
                       const GemmArgs args) {
  using C = Cfg<BN, BKB, SPLIT, EPI>;
  constexpr int S = C::kStages;
  constexpr int NB = C::kAccBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage st: [x -> hi][lo][W_hi][W_lo]; then 8 epilogue staging tiles; then barriers
  uint8_t* store_smem = smem + S * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(store_smem + kStoreBytes);
  // full: TMA landed, one barrier per stage and k-block parity. The two split groups take alternate k-blocks; with
  // an odd stage count a stage's consecutive uses alternate between the groups, and a group waiting on a shared
  // barrier for its next use (two phases on) could pass on the other group's phase still pending (a parity wait
  // cannot tell two phases apart). With one barrier per (stage, parity) each waits only on its own uses, in order.
  uint64_t* full = bars;               // TMA landed            (1 arrival + tx bytes) x 2S
  uint64_t* ready = bars + 2 * S;      // x split done          (4 arrivals)
  uint64_t* empty = bars + 3 * S;      // MMAs of stage done    (1 commit)
  uint64_t* acc_full = bars + 4 * S;   // accumulator complete  (1 commit) x NB
  uint64_t* acc_empty = acc_full + 2;  // accumulator drained   (4 arrivals) x NB
  uint64_t* mma_done = acc_empty + 2;  // teardown drain        (1 commit)
  uint64_t* a_empty = mma_done + 1;    // TMEM A slot free      (1 commit) x 4
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_empty + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // EPI_LN: row statistics (see kLnStatBytes)
  float2* pair_stats = reinterpret_cast<float2*>(store_smem + kStoreBytes + kBarBytes);
  float2* peer_stats = pair_stats + 2 * 2 * 128;
  uint64_t* peer_bar = reinterpret_cast<uint64_t*>(peer_stats + 2 * 128);
  uint64_t* pair_bar = peer_bar + 2;
  uint64_t* load_bar = pair_bar + 4;
  // EPI_LN: the CTA's BN columns never change (tiles are row blocks), so their bias, scale (1 when absent),
  // gamma and beta are read from global memory once, here, and by the epilogue from shared memory
  float* ln_par = reinterpret_cast<float*>(store_smem + kStoreBytes + kBarBytes + 6400);  // [4][BN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TileSched<EPI> ts(args, BN);
  const int num_tiles = ts.count;
  const bool clustered = EPI == EPI_LN && args.cs > 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[2 * s], 1);
      mbar_init(&full[2 * s + 1], 1);
      mbar_init(&ready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);
    }
    mbar_init(mma_done, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&a_empty[q], 1);
    if (EPI == EPI_LN) {
      mbar_init(&peer_bar[0], 128);  // one arrival per lane of the peer's four first-half epilogue warps
      mbar_init(&peer_bar[1], 128);
      for (int q = 0; q < 4; ++q) mbar_init(&pair_bar[q], 64);  // every thread of the two warps of a quadrant
      for (int w = 0; w < 8 * C::kStgTiles; ++w) mbar_init(&load_bar[w], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_whi);
    prefetch_tmap(&map_wlo);
    prefetch_tmap(&map_out);
    if (EPI == EPI_LN) {
      prefetch_tmap(&map_v);
      prefetch_tmap(&map_r);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (EPI == EPI_LN) {
    for (int i = threadIdx.x; i < BN; i += blockDim.x) {
      const int col = ts.col0 + i;
      ln_par[i] = args.bias ? args.bias[col] : 0.f;
      ln_par[BN + i] = args.scale ? args.scale[col] : 1.f;
      ln_par[2 * BN + i] = args.gamma[col];
      ln_par[3 * BN + i] = args.beta[col];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (clustered) cluster_sync();  // the peer's barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t issued[2 * S];
#pragma unroll
      for (int s = 0; s < 2 * S; ++s) issued[s] = 0;
      int st = 0;
      uint32_t phase = 0;
      uint32_t it = 0;  // running k-block index
      bool ok = true;
      for (int tile = ts.first; tile < num_tiles && ok; tile += ts.step) {
        const int m0 = ts.m0(tile), n0 = ts.n0(tile, BN);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&empty[st], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sbase = smem + st * C::kStageBytes;
          const int fb = 2 * st + static_cast<int>(it & 1u);
          uint64_t* fbar = &full[fb];
          mbar_arrive_expect_tx(fbar, C::kTxBytes);
          if (args.conv_c > 0) {
            const int cpb = args.conv_c / C::kBK;  // k-blocks per tap
            const int tap = kb / cpb;
            tma_load_2d(&map_x, fbar, sbase, (kb - tap * cpb) * C::kBK,
                        m0 + (tap / 3 - 1) * args.conv_w + (tap % 3 - 1));
          } else {
            tma_load_2d(&map_x, fbar, sbase, kb * C::kBK, m0);
          }
          constexpr uint32_t kWoff = (C::kTSA ? 1 : 2) * C::kATileBytes;  // W after x (and x_lo, unless TSA)
          tma_load_2d(&map_whi, fbar, sbase + kWoff, kb * C::kBK, n0);
          tma_load_2d(&map_wlo, fbar, sbase + kWoff + C::kBTileBytes, kb * C::kBK, n0);
#pragma unroll
          for (int s = 0; s < 2 * S; ++s) issued[s] += (s == fb);
          ++it;
          if (++st == S) {
            st = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every load this thread issued must have landed before the CTA may exit.
#pragma unroll
      for (int s = 0; s < 2 * S; ++s) {
        if (issued[s] == 0) continue;
        volatile int never = 0;
        if (!mbar_wait(&full[s], (issued[s] - 1) & 1u, &never)) *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop with the same values in every lane; one elected lane issues each MMA.
    {
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      int st = 0;
      uint32_t phase = 0;
      int local = 0;
      uint32_t kit = 0;  // running k-block index: A slot kit % 4
      bool ok = true;
      const uint32_t sb = smem_addr(smem);
      for (int tile = ts.first; tile < num_tiles && ok; tile += ts.step, ++local) {
        const int as = local % NB;
        const uint32_t acc_phase = (local / NB) & 1u;
        if (!mbar_wait_warp(&acc_empty[as], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_main = tmem_base + as * C::kAccCols;
        const uint32_t d_corr = SPLIT ? d_main + BN : d_main;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait_warp(&ready[st], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = sb + st * C::kStageBytes;
          const uint32_t a_lo = a_hi + C::kATileBytes;
          const uint32_t b_hi = a_hi + (C::kTSA ? 1 : 2) * C::kATileBytes;
          const uint32_t b_lo = b_hi + C::kBTileBytes;
          if constexpr (C::kTSA) {  // A_hi / A_lo in this stage's TMEM slot
            const uint32_t aslot = tmem_base + C::kAOffCol + (kit & 3u) * C::kASlotCols;
#pragma unroll
            for (int k = 0; k < C::kBK / 8; ++k) {
              const uint32_t koff = k * 32;
              const uint32_t first = (kb == 0 && k == 0) ? 0u : 1u;
              mma_tf32_ts_w(d_corr, aslot + C::kBK + 8 * k, desc_k<C::kLayout, C::kSbo>(b_hi + koff), idesc, first);
              mma_tf32_ts_w(d_corr, aslot + 8 * k, desc_k<C::kLayout, C::kSbo>(b_lo + koff), idesc, 1u);
              mma_tf32_ts_w(d_main, aslot + 8 * k, desc_k<C::kLayout, C::kSbo>(b_hi + koff), idesc,
                            SPLIT ? first : 1u);
            }
          } else
#pragma unroll
          for (int k = 0; k < C::kBK / 8; ++k) {
            const uint32_t koff = k * 32;  // 8 tf32 = 32 bytes along the swizzled row
            const uint32_t first = (kb == 0 && k == 0) ? 0u : 1u;
            mma_tf32_w(d_corr, desc_k<C::kLayout, C::kSbo>(a_lo + koff), desc_k<C::kLayout, C::kSbo>(b_hi + koff),
                     idesc, first);
            mma_tf32_w(d_corr, desc_k<C::kLayout, C::kSbo>(a_hi + koff), desc_k<C::kLayout, C::kSbo>(b_lo + koff),
                     idesc, 1u);
            mma_tf32_w(d_main, desc_k<C::kLayout, C::kSbo>(a_hi + koff), desc_k<C::kLayout, C::kSbo>(b_hi + koff),
                     idesc, SPLIT ? first : 1u);
          }
          mma_commit_w(&empty[st]);
          if constexpr (C::kTSA) mma_commit_w(&a_empty[kit & 3u]);
          ++kit;
          if (++st == S) {
            st = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_w(&acc_full[as]);
      }
      // Drain: wait for every MMA this warp issued before TMEM is released.
      mma_commit_w(mma_done);
      volatile int never = 0;
      if (!mbar_wait_warp(mma_done, 0, &never)) *abort_flag = 1;
    }
  } else if (warp < kEpilogueWarp0) {
    // ---------------- x split: hi in place, lo alongside ----------------
    // Group g (warps 2-5 or 6-9) takes the k-blocks whose running index has parity g, so two stages are
    // split at once and each group has two MMA k-blocks of time per stage.
    const int group = (warp - kTransformWarp0) >> 2;
    const int t = (threadIdx.x - kTransformWarp0 * 32) & 127;  // 0..127 within the group
    constexpr int kPer = static_cast<int>(C::kATileBytes / 16 / 128);  // float4 of the tile per thread
    constexpr int kRowF4 = BKB / 16;                                    // float4 per tile row
    const bool conv = args.conv_c > 0;
    int st = 0;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = ts.first; tile < num_tiles && ok; tile += ts.step) {
      // implicit convolution: image coordinates of the rows this thread splits (fixed for the tile)
      int py[kPer], px[kPer];
      if (conv) {
        const int m0 = ts.m0(tile), hw = args.conv_h * args.conv_w;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int rem = (m0 + (t + i * 128) / kRowF4) % hw;
          py[i] = rem / args.conv_w;
          px[i] = rem - py[i] * args.conv_w;
        }
      }
      for (int kb = 0; kb < args.k_blocks; ++kb, ++it) {
        if ((it & 1u) == static_cast<uint32_t>(group)) {
          if (!mbar_wait(&full[2 * st + group], (it / C::kFullPeriod) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          int dy = 0, dx = 0;
          if (conv) {
            const int tap = kb / (args.conv_c / C::kBK);
            dy = tap / 3 - 1;
            dx = tap % 3 - 1;
          }
          if constexpr (C::kTSA) {
            // A into TMEM: this warp takes its lane quadrant's 32 rows (row = quad * 32 + lane), reads the row's
            // 16 fp32 from the 64-byte-swizzled tile (chunk c of row r at ((c ^ ((r >> 1) & 3)) << 4)), splits
            // them and stores hi and lo into TMEM slot it % 4, once the MMAs of k-block it - 4 are done with it.
            const int quad = warp & 3, row = quad * 32 + lane;
            if (!mbar_wait(&a_empty[it & 3u], ((it >> 2) & 1u) ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            bool keep = true;
            if (conv) {
              const int rem = (ts.m0(tile) + row) % (args.conv_h * args.conv_w);
              const int yy = rem / args.conv_w + dy, xx = rem % args.conv_w + dx;
              keep = yy >= 0 && yy < args.conv_h && xx >= 0 && xx < args.conv_w;
            }
            const uint8_t* xrow = smem + st * C::kStageBytes + row * 64;
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float4 f = *reinterpret_cast<const float4*>(xrow + ((c ^ ((row >> 1) & 3)) << 4));
              if (!keep) f = make_float4(0.f, 0.f, 0.f, 0.f);
              const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float hv = __uint_as_float(f32_to_tf32_rna(fv[e]));
                hi[4 * c + e] = __float_as_uint(hv);
                lo[4 * c + e] = f32_to_tf32_rna(fv[e] - hv);
              }
            }
            const uint32_t ta =
                tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + C::kAOffCol + (it & 3u) * C::kASlotCols;
            tmem_store_x16(ta, hi);
            tmem_store_x16(ta + C::kBK, lo);
            tmem_store_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[st]);
          } else {
          float4* xa = reinterpret_cast<float4*>(smem + st * C::kStageBytes);
          float4* xl = reinterpret_cast<float4*>(smem + st * C::kStageBytes + C::kATileBytes);
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int idx = t + i * 128;
            float4 v = xa[idx];
            if (conv) {
              const int yy = py[i] + dy, xx = px[i] + dx;
              if (yy < 0 || yy >= args.conv_h || xx < 0 || xx >= args.conv_w) v = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float4 hi, lo;
            hi.x = __uint_as_float(f32_to_tf32_rna(v.x));
            hi.y = __uint_as_float(f32_to_tf32_rna(v.y));
            hi.z = __uint_as_float(f32_to_tf32_rna(v.z));
            hi.w = __uint_as_float(f32_to_tf32_rna(v.w));
            lo.x = __uint_as_float(f32_to_tf32_rna(v.x - hi.x));
            lo.y = __uint_as_float(f32_to_tf32_rna(v.y - hi.y));
            lo.z = __uint_as_float(f32_to_tf32_rna(v.z - hi.z));
            lo.w = __uint_as_float(f32_to_tf32_rna(v.w - hi.w));
            xa[idx] = hi;
            xl[idx] = lo;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ready[st]);
          }
        }
        if (++st == S) st = 0;
      }
    }
  } else if constexpr (EPI == EPI_LN) {
    // ---------------- epilogue: residual + LayerNorm over whole rows ----------------
    // Thread (quad, lane) of warp pair `quad` owns row quad*32 + lane of the tile; half h takes the 32-column
    // chunks c with c % 2 == h, each through the warp's 32x32 staging tile (128-byte swizzle, the layout of the
    // TMA maps). Pass 1 per chunk: the residual chunk comes in by TMA while the accumulator (+ correction) is
    // read from TMEM; v = resid + (acc + bias) * scale; running (mean, M2) of the thread's values; v is stored
    // (if asked) and kept for pass 2 — in TMEM over the accumulator, or, with a single accumulator buffer and v
    // stored, in the output itself (the accumulator is then released right after pass 1, so the next tile's MMAs
    // overlap the rest). The two halves combine their statistics in shared memory, the CTAs of a cluster swap
    // theirs through distributed shared memory (each combines in rank order, so every CTA derives bit-identical
    // mean and rstd for a row), and pass 2 stores act((v - mean) * rstd * gamma + beta).
    const int quad = warp & 3;
    const int half = (warp - kEpilogueWarp0) >> 2;
    const int ew = warp - kEpilogueWarp0;
    const int row_t = quad * 32 + lane;
    uint8_t* stile = store_smem + ew * kStoreTileBytes;
    uint64_t* lbar = &load_bar[ew];
    uint32_t lphase = 0;
    const uint32_t peer = clustered ? (cluster_ctarank() ^ 1u) : 0u;
    const bool rank0 = !clustered || cluster_ctarank() == 0;
    const bool v_global = NB == 1 && args.write_v;
    const float n_half = static_cast<float>(BN / 2);
    const float inv_n = 1.0f / static_cast<float>(args.N);
    bool ok = true;
    // Loads one 32x32 chunk (rows m0 + quad*32.., columns col0..) of `map` into the staging tile, once the
    // previous bulk operation of this warp on the tile is complete. Returns false if the wait runs out.
    auto load_chunk = [&](const CUtensorMap* map, int col0, int row0) -> bool {
      if (lane == 0) bulk_wait<0>();
      __syncwarp();
      fence_proxy_async_smem();
      if (lane == 0) {
        mbar_arrive_expect_tx(lbar, kStoreTileBytes);
        tma_load_2d(map, lbar, stile, col0, row0);
      }
      const bool done = mbar_wait(lbar, lphase, abort_flag);
      lphase ^= 1u;
      return done;
    };
    if constexpr (C::kStgTiles == 2) {
      // Two staging tiles per warp (no correction accumulator, so v stays in tensor memory between the passes).
      // A running chunk count gk picks the tile (gk & 1). Pass 1 issues the next chunk's residual load into the
      // other tile before it waits for and works on this chunk's, so each residual read overlaps the previous
      // chunk; before a tile is loaded or written, the bulk stores issued from it have read it (the newest
      // store may stay pending when it came from the other tile).
      uint8_t* const stl[2] = {stile, store_smem + C::kStg2Off + ew * kStoreTileBytes};
      uint64_t* const lbr[2] = {&load_bar[ew], &load_bar[8 + ew]};
      uint32_t lph[2] = {0u, 0u};
      uint32_t gk = 0;
      int newest = -1;  // tile of this warp's newest bulk store (-1: none)
      auto free_tile = [&](int b) {
        if (lane == 0) {
          if (newest == b) bulk_wait_read<0>();
          else if (newest >= 0) bulk_wait_read<1>();
        }
        __syncwarp();
      };
      auto load_resid = [&](int b, int col0, int row0) {
        free_tile(b);
        fence_proxy_async_smem();
        if (lane == 0) {
          mbar_arrive_expect_tx(lbr[b], kStoreTileBytes);
          tma_load_2d(&map_r, lbr[b], stl[b], col0, row0);
        }
      };
      auto store_tile = [&](const CUtensorMap* map, int b, int col0, int row0) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(map, stl[b], col0, row0);
          bulk_commit();
        }
        newest = b;
      };
      constexpr int kChunks = BN / 64;  // this warp's 32-column chunks of a tile (c = half, half + 2, ...)
      int local = 0;
      for (int tile = ts.first; tile < num_tiles && ok; tile += ts.step, ++local) {
        const int as = local % NB;
        const uint32_t acc_phase = (local / NB) & 1u;
        if (!mbar_wait(&acc_full[as], acc_phase, abort_flag)) break;
        tc_fence_after();
        const int m0 = ts.m0(tile), n0 = ts.n0(tile, BN);
        const int row0 = m0 + quad * 32;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + as * C::kAccCols;
        if (args.resid && tile + ts.step < num_tiles) {  // the residual slices of this thread's next row into L2
          const int64_t nrow = static_cast<int64_t>(ts.m0(tile + ts.step)) + row_t;
          if (nrow < args.M)
            for (int c = half; c < BN / 32; c += 2) {
              const float* p = args.resid + nrow * args.N + n0 + c * 32;
              asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
              asm volatile("prefetch.global.L2 [%0];" ::"l"(p + 31));
            }
        }
        float2 st = make_float2(0.f, 0.f);  // (mean, M2) of the values seen so far
        float cnt = 0.f;
        if (args.resid) load_resid(static_cast<int>(gk & 1u), n0 + half * 32, row0);
#pragma unroll 1
        for (int ci = 0; ci < kChunks; ++ci) {
          const int c = half + 2 * ci;
          const int col0 = n0 + c * 32;
          const int b = static_cast<int>(gk & 1u);
          if (args.resid && ci + 1 < kChunks) load_resid(b ^ 1, col0 + 64, row0);  // the next chunk's residual
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_ld_wait_regs(r);
          if (args.resid) {
            ok = mbar_wait(lbr[b], lph[b], abort_flag);
            lph[b] ^= 1u;
            if (!ok) break;
          } else {
            free_tile(b);  // v is staged in this tile below
          }
          uint8_t* sb = stl[b];
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = col0 + 4 * j;
            float4* slot = reinterpret_cast<float4*>(sb + lane * 128 + ((j ^ (lane & 7)) << 4));
            const float4 hv = args.resid ? *slot : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 bb = *reinterpret_cast<const float4*>(ln_par + (col - ts.col0));
            const float4 sc = *reinterpret_cast<const float4*>(ln_par + BN + (col - ts.col0));
            float4 v;
            v.x = hv.x + (__uint_as_float(r[4 * j + 0]) + bb.x) * sc.x;
            v.y = hv.y + (__uint_as_float(r[4 * j + 1]) + bb.y) * sc.y;
            v.z = hv.z + (__uint_as_float(r[4 * j + 2]) + bb.z) * sc.z;
            v.w = hv.w + (__uint_as_float(r[4 * j + 3]) + bb.w) * sc.w;
            r[4 * j + 0] = __float_as_uint(v.x);
            r[4 * j + 1] = __float_as_uint(v.y);
            r[4 * j + 2] = __float_as_uint(v.z);
            r[4 * j + 3] = __float_as_uint(v.w);
            sum += (v.x + v.y) + (v.z + v.w);
            if (args.write_v) *slot = v;
          }
          const float cm = sum * (1.0f / 32.0f);
          float m2 = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float d = __uint_as_float(r[j]) - cm;
            m2 += d * d;
          }
          if (cnt == 0.f) {
            st = make_float2(cm, m2);
          } else {  // Chan: (cnt values) + (32 values)
            const float tot = cnt + 32.f;
            const float d = cm - st.x;
            st.x += d * (32.f / tot);
            st.y += m2 + d * d * (cnt * 32.f / tot);
          }
          cnt += 32.f;
          tmem_store_x32(taddr + c * 32, r);
          if (args.write_v) store_tile(&map_v, b, col0, row0);
          ++gk;
        }
        if (!ok) break;
        tmem_store_wait();
        // Combine the two halves of the row (same order in both warps of the pair).
        const int par = local & 1;
        pair_stats[(par * 2 + half) * 128 + row_t] = st;
        mbar_arrive(&pair_bar[quad]);
        if (!mbar_wait(&pair_bar[quad], local & 1, abort_flag)) break;
        st = combine_stats(pair_stats[(par * 2 + 0) * 128 + row_t], pair_stats[(par * 2 + 1) * 128 + row_t], n_half);
        if (clustered) {
          if (half == 0) {
            const uint32_t dst = cluster_map(smem_addr(&peer_stats[par * 128 + row_t]), peer);
            cluster_store_f2(dst, st.x, st.y);
            mbar_arrive_cluster(cluster_map(smem_addr(&peer_bar[par]), peer));
          }
          if (!mbar_wait_cluster(&peer_bar[par], (local >> 1) & 1, abort_flag)) break;
          const float2 other = peer_stats[par * 128 + row_t];
          st = rank0 ? combine_stats(st, other, static_cast<float>(BN)) : combine_stats(other, st, static_cast<float>(BN));
        }
        const float mean = st.x;
        const float rstd = 1.0f / sqrtf(st.y * inv_n + args.eps);
#pragma unroll 1
        for (int ci = 0; ci < kChunks; ++ci) {
          const int c = half + 2 * ci;
          const int col0 = n0 + c * 32;
          const int b = static_cast<int>(gk & 1u);
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_ld_wait_regs(r);
          if (ci + 1 == kChunks) {  // this warp's last read of the tile: release the accumulator
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[as]);
          }
          free_tile(b);
          uint8_t* sb = stl[b];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = col0 + 4 * j;
            const float4 g = *reinterpret_cast<const float4*>(ln_par + 2 * BN + (col - ts.col0));
            const float4 bt = *reinterpret_cast<const float4*>(ln_par + 3 * BN + (col - ts.col0));
            float4 o;
            o.x = ln_act((__uint_as_float(r[4 * j + 0]) - mean) * rstd * g.x + bt.x, args.act);
            o.y = ln_act((__uint_as_float(r[4 * j + 1]) - mean) * rstd * g.y + bt.y, args.act);
            o.z = ln_act((__uint_as_float(r[4 * j + 2]) - mean) * rstd * g.z + bt.z, args.act);
            o.w = ln_act((__uint_as_float(r[4 * j + 3]) - mean) * rstd * g.w + bt.w, args.act);
            *reinterpret_cast<float4*>(sb + lane * 128 + ((j ^ (lane & 7)) << 4)) = o;
          }
          store_tile(&map_out, b, col0, row0);
          ++gk;
        }
      }
    } else {
    int local = 0;
    for (int tile = ts.first; tile < num_tiles && ok; tile += ts.step, ++local) {
      const int as = local % NB;
      const uint32_t acc_phase = (local / NB) & 1u;
      if (!mbar_wait(&acc_full[as], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int m0 = ts.m0(tile), n0 = ts.n0(tile, BN);
      const int row0 = m0 + quad * 32;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + as * C::kAccCols;
      if (args.resid && tile + ts.step < num_tiles) {  // the residual slices of this thread's next row into L2
        const int64_t nrow = static_cast<int64_t>(ts.m0(tile + ts.step)) + row_t;
        if (nrow < args.M)
          for (int c = half; c < BN / 32; c += 2) {
            const float* p = args.resid + nrow * args.N + n0 + c * 32;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p + 31));
          }
      }
      float2 st = make_float2(0.f, 0.f);  // (mean, M2) of the values seen so far
      float cnt = 0.f;
#pragma unroll 1
      for (int c = half; c < BN / 32; c += 2) {
        const int col0 = n0 + c * 32;
        if (args.resid) {
          if (lane == 0) bulk_wait_read<0>();  // the previous store from the staging tile has read it
          __syncwarp();
          fence_proxy_async_smem();
          if (lane == 0) {
            mbar_arrive_expect_tx(lbar, kStoreTileBytes);
            tma_load_2d(&map_r, lbar, stile, col0, row0);
          }
        } else {
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        if constexpr (SPLIT) {
          uint32_t q[32];
          tmem_ld_32x32b_x32(taddr + BN + c * 32, q);
          tmem_ld_wait_regs(r);
          tmem_ld_wait_regs(q);
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
        } else {
          tmem_ld_wait_regs(r);
        }
        if (args.resid) {
          ok = mbar_wait(lbar, lphase, abort_flag);
          lphase ^= 1u;
          if (!ok) break;
        }
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = col0 + 4 * j;
          float4* slot = reinterpret_cast<float4*>(stile + lane * 128 + ((j ^ (lane & 7)) << 4));
          const float4 hv = args.resid ? *slot : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 b = *reinterpret_cast<const float4*>(ln_par + (col - ts.col0));
          const float4 sc = *reinterpret_cast<const float4*>(ln_par + BN + (col - ts.col0));
          float4 v;
          v.x = hv.x + (__uint_as_float(r[4 * j + 0]) + b.x) * sc.x;
          v.y = hv.y + (__uint_as_float(r[4 * j + 1]) + b.y) * sc.y;
          v.z = hv.z + (__uint_as_float(r[4 * j + 2]) + b.z) * sc.z;
          v.w = hv.w + (__uint_as_float(r[4 * j + 3]) + b.w) * sc.w;
          r[4 * j + 0] = __float_as_uint(v.x);
          r[4 * j + 1] = __float_as_uint(v.y);
          r[4 * j + 2] = __float_as_uint(v.z);
          r[4 * j + 3] = __float_as_uint(v.w);
          sum += (v.x + v.y) + (v.z + v.w);
          if (args.write_v) *slot = v;
        }
        const float cm = sum * (1.0f / 32.0f);
        float m2 = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = __uint_as_float(r[j]) - cm;
          m2 += d * d;
        }
        if (cnt == 0.f) {
          st = make_float2(cm, m2);
        } else {  // Chan: (cnt values) + (32 values)
          const float tot = cnt + 32.f;
          const float d = cm - st.x;
          st.x += d * (32.f / tot);
          st.y += m2 + d * d * (cnt * 32.f / tot);
        }
        cnt += 32.f;
        if (!v_global) tmem_store_x32(taddr + c * 32, r);
        if (args.write_v) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_v, stile, col0, row0);
            bulk_commit();
          }
        }
      }
      if (!ok) break;
      if (v_global) {  // v lives in the output now: hand the accumulator back to the MMAs
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[as]);
      } else {
        tmem_store_wait();
      }
      // Combine the two halves of the row (same order in both warps of the pair).
      const int par = local & 1;
      pair_stats[(par * 2 + half) * 128 + row_t] = st;
      mbar_arrive(&pair_bar[quad]);
      if (!mbar_wait(&pair_bar[quad], local & 1, abort_flag)) break;
      st = combine_stats(pair_stats[(par * 2 + 0) * 128 + row_t], pair_stats[(par * 2 + 1) * 128 + row_t], n_half);
      if (clustered) {
        if (half == 0) {
          const uint32_t dst = cluster_map(smem_addr(&peer_stats[par * 128 + row_t]), peer);
          cluster_store_f2(dst, st.x, st.y);
          mbar_arrive_cluster(cluster_map(smem_addr(&peer_bar[par]), peer));
        }
        if (!mbar_wait_cluster(&peer_bar[par], (local >> 1) & 1, abort_flag)) break;
        const float2 other = peer_stats[par * 128 + row_t];
        st = rank0 ? combine_stats(st, other, static_cast<float>(BN)) : combine_stats(other, st, static_cast<float>(BN));
      }
      const float mean = st.x;
      const float rstd = 1.0f / sqrtf(st.y * inv_n + args.eps);
#pragma unroll 1
      for (int c = half; c < BN / 32; c += 2) {
        const int col0 = n0 + c * 32;
        uint32_t r[32];
        if (v_global) {
          // v of this chunk was stored by this warp in pass 1; bulk_wait<0> inside load_chunk makes that store
          // complete before the load is issued
          if (!(ok = load_chunk(&map_v, col0, row0))) break;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(stile + lane * 128 + ((j ^ (lane & 7)) << 4));
            r[4 * j + 0] = __float_as_uint(v.x);
            r[4 * j + 1] = __float_as_uint(v.y);
            r[4 * j + 2] = __float_as_uint(v.z);
            r[4 * j + 3] = __float_as_uint(v.w);
          }
        } else {
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_ld_wait_regs(r);
          if (c + 2 >= BN / 32) {  // this warp's last read of the tile: release the accumulator
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[as]);
          }
          if (lane == 0) bulk_wait_read<0>();
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = col0 + 4 * j;
          const float4 g = *reinterpret_cast<const float4*>(ln_par + 2 * BN + (col - ts.col0));
          const float4 bt = *reinterpret_cast<const float4*>(ln_par + 3 * BN + (col - ts.col0));
          float4 o;
          o.x = ln_act((__uint_as_float(r[4 * j + 0]) - mean) * rstd * g.x + bt.x, args.act);
          o.y = ln_act((__uint_as_float(r[4 * j + 1]) - mean) * rstd * g.y + bt.y, args.act);
          o.z = ln_act((__uint_as_float(r[4 * j + 2]) - mean) * rstd * g.z + bt.z, args.act);
          o.w = ln_act((__uint_as_float(r[4 * j + 3]) - mean) * rstd * g.w + bt.w, args.act);
          *reinterpret_cast<float4*>(stile + lane * 128 + ((j ^ (lane & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_out, stile, col0, row0);
          bulk_commit();
        }
      }
    }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    // Warp pair per TMEM lane quadrant; half h of the pair takes the 32-column chunks c with c % 2 == h. Each
    // chunk: tcgen05.ld of the main (and correction) accumulator, + bias, activation, a 128-byte-swizzled 32x32
    // tile in shared memory, and one TMA store (rows >= M and columns >= N are clipped by the tensor map).
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = (warp - kEpilogueWarp0) >> 2;
    uint8_t* stile = store_smem + (warp - kEpilogueWarp0) * kStoreTileBytes;
    int local = 0;
    for (int tile = ts.first; tile < num_tiles; tile += ts.step, ++local) {
      const int as = local % NB;
      const uint32_t acc_phase = (local / NB) & 1u;
      if (!mbar_wait(&acc_full[as], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int m0 = ts.m0(tile), n0 = ts.n0(tile, BN);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + as * C::kAccCols;
#pragma unroll 1
      for (int c = half; c < BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        if constexpr (SPLIT) {
          uint32_t q[32];
          tmem_ld_32x32b_x32(taddr + BN + c * 32, q);
          tmem_ld_wait_regs(r);
          tmem_ld_wait_regs(q);
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
        } else {
          tmem_ld_wait_regs(r);
        }
        if (c + 2 >= BN / 32) {  // this warp's last chunk of the tile: release the accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[as]);
        }
        const int col0 = n0 + c * 32;
        // the previous TMA store from this warp's tile must have finished reading it
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = col0 + 4 * j;
          float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
          if (args.bias && col < args.N) b = __ldg(reinterpret_cast<const float4*>(args.bias + col));
          float4 ad = make_float4(0.f, 0.f, 0.f, 0.f);
          if (args.addend) {
            const int row = m0 + quad * 32 + lane;
            if (row < args.M && col < args.add_cols)
              ad = __ldg(reinterpret_cast<const float4*>(args.addend + static_cast<int64_t>(row) * args.ld_add + col));
          }
          float4 o;
          o.x = apply_act(__uint_as_float(r[4 * j + 0]) + b.x + ad.x, args.act);
          o.y = apply_act(__uint_as_float(r[4 * j + 1]) + b.y + ad.y, args.act);
          o.z = apply_act(__uint_as_float(r[4 * j + 2]) + b.z + ad.z, args.act);
          o.w = apply_act(__uint_as_float(r[4 * j + 3]) + b.w + ad.w, args.act);
          // row `lane` of the tile, 16-byte chunk j, 128-byte swizzle: chunk position j ^ (row % 8)
          *reinterpret_cast<float4*>(stile + lane * 128 + ((j ^ (lane & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_out, stile, col0, m0 + quad * 32);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();  // all stores complete before the CTA exits
    __syncwarp();
  }

  __syncwarp();
  if (clustered) cluster_sync();  // no CTA leaves while its peer may still write into its shared memory
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && args.dev_status) atomicExch(args.dev_status, KO_ERR_DEVICE_TIMEOUT);
}

// W[K][N] -> packed[2][N][K] (hi = tf32_rn(w), lo = tf32_rn(w - hi)), transposed through a 32x32 tile.
__global__ void __launch_bounds__(256) pack_weight_kernel(const float* __restrict__ w, int K, int N,
                                                          float* __restrict__ packed) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    tile[i][threadIdx.x] = (k < K && n < N) ? w[static_cast<int64_t>(k) * N + n] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < K) {
      const float v = tile[threadIdx.x][i];
      const float hi = __uint_as_float(kodev::f32_to_tf32_rna(v));
      const float lo = __uint_as_float(kodev::f32_to_tf32_rna(v - hi));
      packed[static_cast<int64_t>(n) * K + k] = hi;
      packed[static_cast<int64_t>(N) * K + static_cast<int64_t>(n) * K + k] = lo;
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------------------
namespace {

template <int BN, int BKB, bool SPLIT>
int launch_gemm(const float* x, const float* w_packed, const float* bias, const float* addend, int64_t ld_add,
                int64_t add_cols, int64_t M, int64_t K, int64_t N, int act, float* out, int* dev_status,
                cudaStream_t stream) {
  using C = Cfg<BN, BKB, SPLIT, EPI_ACT>;
  const CUtensorMapSwizzle sw = BKB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap mx, mhi, mlo;
  int st = ko::make_tmap_2d_f32(&mx, x, M, K, K, BM, C::kBK, sw, "ko_linear x");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&mhi, w_packed, N, K, K, BN, C::kBK, sw, "ko_linear w_hi");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&mlo, w_packed + N * K, N, K, K, BN, C::kBK, sw, "ko_linear w_lo");
  if (st) return st;
  CUtensorMap mout;
  st = ko::make_tmap_2d_f32(&mout, out, M, N, N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, "ko_linear out");
  if (st) return st;
  const ko::DeviceInfo* dinfo = nullptr;
  st = ko::device_or_fail(&dinfo, "ko_linear");
  if (st) return st;
  const ko::DeviceInfo& info = *dinfo;
  if (static_cast<int64_t>(C::kSmemBytes) > info.max_smem_optin)
    return ko::fail(KO_ERR_UNSUPPORTED, "ko_linear: not enough shared memory on this device");
  cudaError_t e = cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, BKB, SPLIT, EPI_ACT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::kSmemBytes));
  if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_linear: cudaFuncSetAttribute failed");
  GemmArgs a = {};
  a.bias = bias;
  a.out = out;
  a.dev_status = dev_status;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.act = act;
  a.addend = addend;
  a.ld_add = static_cast<int>(ld_add);
  a.add_cols = static_cast<int>(add_cols);
  a.m_tiles = static_cast<int>((M + BM - 1) / BM);
  a.n_tiles = static_cast<int>((N + BN - 1) / BN);
  a.k_blocks = static_cast<int>((K + C::kBK - 1) / C::kBK);
  const int tiles = a.m_tiles * a.n_tiles;
  const int grid = std::min(tiles, info.sm_count);
  a.cs = 1;
  gemm_tf32x3_kernel<BN, BKB, SPLIT, EPI_ACT><<<grid, kThreads, C::kSmemBytes, stream>>>(mx, mhi, mlo, mout, mout, mout, a);
  return ko::check_launch("ko_linear_f32_packed");
}

// GEMM + residual + LayerNorm: clusters of cs = N / BN CTAs, one row block per cluster at a time.
template <int BN, bool SPLIT>
int launch_gemm_ln(const float* x, const float* w_packed, const float* bias, const float* scale, const float* resid,
                   const float* gamma, const float* beta, float eps, int64_t M, int64_t K, int64_t N, int act,
                   float* v_out, float* y, int* dev_status, cudaStream_t stream, int conv_h = 0, int conv_w = 0,
                   int conv_c = 0, int64_t ldx = 0, int64_t ldy = 0) {
  constexpr int BKB = 64;
  using C = Cfg<BN, BKB, SPLIT, EPI_LN>;
  const int cs = static_cast<int>(N / BN);
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap mx, mhi, mlo, my, mv;
  const int64_t xcols = conv_c > 0 ? conv_c : K;  // an implicit convolution reads x as [M][C]
  if (ldx == 0) ldx = xcols;                       // row pitches of x and y (0: dense rows)
  if (ldy == 0) ldy = N;
  int st = ko::make_tmap_2d_f32(&mx, x, M, xcols, ldx, BM, C::kBK, sw, "ko_linear_residual_ln x");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&mhi, w_packed, N, K, K, BN, C::kBK, sw, "ko_linear_residual_ln w_hi");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&mlo, w_packed + N * K, N, K, K, BN, C::kBK, sw, "ko_linear_residual_ln w_lo");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&my, y, M, N, ldy, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, "ko_linear_residual_ln y");
  if (st) return st;
  st = ko::make_tmap_2d_f32(&mv, v_out ? v_out : y, M, N, N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                            "ko_linear_residual_ln h_out");
  if (st) return st;
  CUtensorMap mr;
  st = ko::make_tmap_2d_f32(&mr, resid ? resid : y, M, N, N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                            "ko_linear_residual_ln resid");
  if (st) return st;
  const ko::DeviceInfo* dinfo = nullptr;
  st = ko::device_or_fail(&dinfo, "ko_linear_residual_ln");
  if (st) return st;
  const ko::DeviceInfo& info = *dinfo;
  if (static_cast<int64_t>(C::kSmemBytes) > info.max_smem_optin)
    return ko::fail(KO_ERR_UNSUPPORTED, "ko_linear_residual_ln: not enough shared memory on this device");
  auto kernel = gemm_tf32x3_kernel<BN, BKB, SPLIT, EPI_LN>;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::kSmemBytes));
  if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_linear_residual_ln: cudaFuncSetAttribute failed");
  GemmArgs a = {};
  a.bias = bias;
  a.out = y;
  a.dev_status = dev_status;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.act = act;
  a.m_tiles = static_cast<int>((M + BM - 1) / BM);
  a.n_tiles = cs;
  a.k_blocks = static_cast<int>((K + C::kBK - 1) / C::kBK);
  a.scale = scale;
  a.resid = resid;
  a.gamma = gamma;
  a.beta = beta;
  a.eps = eps;
  a.write_v = v_out != nullptr;
  a.cs = cs;
  a.conv_h = conv_h;
  a.conv_w = conv_w;
  a.conv_c = conv_c;

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cs);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // As many clusters as fit at once (one CTA per SM; SMs a GPC cannot pair up stay idle), at most one per row
  // block; each cluster then strides over the row blocks.
  static std::atomic<int> max_clusters[2][64];  // per cluster size and device, looked up once
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& slot = max_clusters[cs - 1][dev & 63];
  int mc = slot.load();
  if (mc == 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(info.sm_count / cs * cs));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess || n < 1)
      return ko::fail(e != cudaSuccess ? static_cast<int>(e) : KO_ERR_UNSUPPORTED,
                      "ko_linear_residual_ln: no cluster of this size fits on the device");
    mc = n;
    slot.store(n);
  }
  const int clusters = std::min(a.m_tiles, mc);
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * cs));
  e = cudaLaunchKernelEx(&cfg, kernel, mx, mhi, mlo, my, mv, mr, a);
  if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_linear_residual_ln: launch failed");
  return ko::check_launch("ko_linear_residual_ln_f32_packed");
}

using LaunchFn = int (*)(const float*, const float*, const float*, const float*, int64_t, int64_t, int64_t, int64_t,
                         int64_t, int, float*, int*,
                         cudaStream_t);

struct Variant {
  int bn, bkb, split;
  LaunchFn fn;
};

const Variant kVariants[] = {
    {256, 64, 1, launch_gemm<256, 64, true>},   {256, 64, 0, launch_gemm<256, 64, false>},
    {192, 64, 1, launch_gemm<192, 64, true>},   {192, 64, 0, launch_gemm<192, 64, false>},
    {128, 64, 1, launch_gemm<128, 64, true>},   {128, 64, 0, launch_gemm<128, 64, false>},
    {256, 128, 1, launch_gemm<256, 128, true>}, {256, 128, 0, launch_gemm<256, 128, false>},
    {128, 128, 1, launch_gemm<128, 128, true>}, {128, 128, 0, launch_gemm<128, 128, false>},
};

// Measurement builds may pin one variant at compile time (-DKO_GEMM_FORCE_VARIANT=bn,bkb,split); the shipped
// library chooses by shape only.
const Variant* forced_variant() {
#ifdef KO_GEMM_FORCE_VARIANT
  static const Variant* v = [] {
    const int want[3] = {KO_GEMM_FORCE_VARIANT};
    for (const Variant& c : kVariants)
      if (c.bn == want[0] && c.bkb == want[1] && c.split == want[2]) return &c;
    return static_cast<const Variant*>(nullptr);
  }();
  return v;
#else
  return nullptr;
#endif
}

// Default choice.
//   Accumulator: the split correction accumulator (SPLIT) only for K > 512. Up to K = 512 the single accumulator
//   stays within 3e-6 of float64 (normwise, N(0,1) activations, K = 384) — inside the 1e-5 bar with room — and
//   leaves TMEM for two accumulator buffers at 256 columns, so the epilogue of one tile overlaps the MMAs of the
//   next. Beyond that its error grows with K (1.1e-5 at K = 1536), and SPLIT keeps it at 4e-6.
//   Tile width: the BN in {256, 192, 128} with the least estimated time, waves x BN x cost per column, where
//   the cost per column (1, 1.04, 1.45 without SPLIT; 1.12, 0.93, 1.45 with it) was measured on B200 at the
//   model's shapes. 192-wide tiles take A from tensor memory (7-10 % faster than with A in shared memory); wider
//   tiles read each x tile for more columns; with SPLIT, 256-wide tiles hold all 512 TMEM columns (one buffer)
//   and lose the overlap of epilogue and MMAs.
#ifndef KO_SPLIT_MIN_K
#define KO_SPLIT_MIN_K 512  // measurement builds may move the threshold (-DKO_SPLIT_MIN_K=0: SPLIT everywhere)
#endif
const Variant* choose_variant(int64_t M, int64_t N, int64_t K, int64_t sms) {
  if (const Variant* f = forced_variant()) return f;
  const int split = K > KO_SPLIT_MIN_K ? 1 : 0;
  const int64_t m_tiles = (M + BM - 1) / BM;
  const int bns[3] = {256, 192, 128};
  const double cost_plain[3] = {1.0, 1.04, 1.45};
  const double cost_split[3] = {1.12, 0.93, 1.45};
  int best = 0;
  double best_t = 0;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = m_tiles * ((N + bns[i] - 1) / bns[i]);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double t = static_cast<double>(waves) * bns[i] * (split ? cost_split[i] : cost_plain[i]);
    if (i == 0 || t < best_t) {
      best = i;
      best_t = t;
    }
  }
  for (const Variant& c : kVariants)
    if (c.bn == bns[best] && c.bkb == 64 && c.split == split) return &c;
  return &kVariants[0];
}

int validate_linear(const float* x, const float* w, const float* bias, int64_t M, int64_t K, int64_t N,
                    const float* out, const char* who) {
  if (M < 0 || K < 4 || N < 4 || K % 4 != 0 || N % 4 != 0 || M > INT32_MAX || K > (1 << 20) || N > (1 << 20))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": need K % 4 == 0 and N % 4 == 0");
  if (M == 0) return KO_OK;
  if (!x || !w || !out) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  if (!ko::aligned16(x) || !ko::aligned16(w) || !ko::aligned16(out) || (bias && !ko::aligned16(bias)))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": pointers must be 16-byte aligned");
  return KO_OK;
}

}  // namespace

extern "C" int64_t ko_linear_workspace_bytes(int64_t K, int64_t N) { return 2 * K * N * 4; }

extern "C" int ko_pack_weight_tf32x3(const float* w, int64_t K, int64_t N, float* w_packed, ko_stream_t stream) {
  if (K < 1 || N < 1 || K > (1 << 20) || N > (1 << 20) || !w || !w_packed)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_pack_weight_tf32x3: bad arguments");
  dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((K + 31) / 32));
  pack_weight_kernel<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, static_cast<int>(K), static_cast<int>(N), w_packed);
  return ko::check_launch("ko_pack_weight_tf32x3");
}

extern "C" int ko_linear_f32_packed(const float* x, const float* w_packed, const float* bias, int64_t M, int64_t K,
                                    int64_t N, int act, float* out, int* dev_status, ko_stream_t stream) {
  int st = validate_linear(x, w_packed, bias, M, K, N, out, "ko_linear_f32_packed");
  if (st || M == 0) return st;
  if (act != KO_ACT_NONE && act != KO_ACT_GELU && act != KO_ACT_RELU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_linear_f32_packed: unknown activation");
  const ko::DeviceInfo* info = nullptr;
  st = ko::device_or_fail(&info, "ko_linear_f32_packed");
  if (st) return st;
  const Variant* v = choose_variant(M, N, K, info->sm_count);
  return v->fn(x, w_packed, bias, nullptr, 0, 0, M, K, N, act, out, dev_status, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ko_linear_add_f32_packed(const float* x, const float* w_packed, const float* bias, const float* addend,
                                        int64_t ld_addend, int64_t add_cols, int64_t M, int64_t K, int64_t N, int act,
                                        float* out, int* dev_status, ko_stream_t stream) {
  const char* who = "ko_linear_add_f32_packed";
  int st = validate_linear(x, w_packed, bias, M, K, N, out, who);
  if (st || M == 0) return st;
  if (act != KO_ACT_NONE && act != KO_ACT_GELU && act != KO_ACT_RELU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": unknown activation");
  if (!addend || !ko::aligned16(addend) || add_cols < 4 || add_cols > N || add_cols % 4 != 0 || ld_addend < add_cols ||
      ld_addend % 4 != 0 || ld_addend > INT32_MAX || M * ld_addend > (int64_t(1) << 40))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": addend must be 16-byte aligned, 4 <= add_cols <= N, "
                                                                "add_cols and ld_addend multiples of 4, ld >= add_cols");
  if (addend == out) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": out must not alias addend");
  const ko::DeviceInfo* info = nullptr;
  st = ko::device_or_fail(&info, who);
  if (st) return st;
  const Variant* v = choose_variant(M, N, K, info->sm_count);
  return v->fn(x, w_packed, bias, addend, ld_addend, add_cols, M, K, N, act, out, dev_status,
               reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ko_linear_residual_ln_f32_packed(const float* x, const float* w_packed, const float* bias,
                                                const float* scale, const float* resid, const float* gamma,
                                                const float* beta, float eps, int64_t M, int64_t K, int64_t N,
                                                int act, float* h_out, float* y, int64_t ldy, int* dev_status,
                                                ko_stream_t stream) {
  const char* who = "ko_linear_residual_ln_f32_packed";
  int st = validate_linear(x, w_packed, bias, M, K, N, y, who);
  if (st || M == 0) return st;
  if (N != 128 && N != 192 && N != 256 && N != 384 && N != 512)
    return ko::fail(KO_ERR_UNSUPPORTED, std::string(who) + ": N must be 128, 192, 256, 384 or 512 (whole rows in "
                                                           "one CTA or a pair of CTAs)");
  if (act != KO_ACT_NONE && act != KO_ACT_SILU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": act must be KO_ACT_NONE or KO_ACT_SILU");
  if (!gamma || !beta || !(eps >= 0.0f))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": gamma and beta are required, eps >= 0");
  if (!ko::aligned16(gamma) || !ko::aligned16(beta) || (scale && !ko::aligned16(scale)) ||
      (resid && !ko::aligned16(resid)) || (h_out && !ko::aligned16(h_out)))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": pointers must be 16-byte aligned");
  if (y == resid || y == h_out || y == x)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": y must not alias x, resid or h_out");
  if (ldy != 0 && (ldy < N || ldy % 4 != 0 || ldy > INT32_MAX))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": ldy must be 0 or a multiple of 4 >= N");
  const ko::DeviceInfo* info = nullptr;
  st = ko::device_or_fail(&info, who);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool split = K > KO_SPLIT_MIN_K;
  // N = 256 rows fit one 256-wide CTA or a cluster of two 128-wide ones. With fewer row blocks than two per SM
  // (the decoder's 300 queries per frame), the pair halves each row block's time and wins (fc2, K = 2048: 225 ->
  // 196 us at 64 frames); with many row blocks the single CTA keeps its wider tile (158 against 185 us at 102400
  // rows, K = 384).
  const int64_t m_tiles = (M + BM - 1) / BM;
  const int bn = N == 384 ? 192
                 : N == 512 ? 256
                 : (N == 256 && m_tiles < 2 * static_cast<int64_t>(info->sm_count)) ? 128
                                                                                                : static_cast<int>(N);
#define KO_LN_CASE(BNV)                                                                                         \
  if (bn == BNV)                                                                                               \
    return split ? launch_gemm_ln<BNV, true>(x, w_packed, bias, scale, resid, gamma, beta, eps, M, K, N, act,   \
                                             h_out, y, dev_status, s, 0, 0, 0, 0, ldy)                         \
                 : launch_gemm_ln<BNV, false>(x, w_packed, bias, scale, resid, gamma, beta, eps, M, K, N, act,  \
                                              h_out, y, dev_status, s, 0, 0, 0, 0, ldy);
  KO_LN_CASE(128)
  KO_LN_CASE(192)
  KO_LN_CASE(256)
#undef KO_LN_CASE
  return ko::fail(KO_ERR_UNSUPPORTED, std::string(who) + ": no tile for this N");
}

extern "C" int ko_conv3x3_ln_f32_packed(const float* x, int64_t ldx, const float* w_packed, const float* bias,
                                        const float* gamma, const float* beta, float eps, int64_t B, int64_t H,
                                        int64_t W, int64_t C, int64_t N, int act, float* y, int64_t ldy,
                                        int* dev_status, ko_stream_t stream) {
  const char* who = "ko_conv3x3_ln_f32_packed";
  if (B < 0 || H < 1 || W < 1 || C < 16 || C % 16 != 0 || B * H * W > INT32_MAX || C > 4096)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": need C % 16 == 0 and a batch below 2^31 pixels");
  const int64_t M = B * H * W, K = 9 * C;
  int st = validate_linear(x, w_packed, bias, M, K, N, y, who);
  if (st || M == 0) return st;
  if (N != 128 && N != 192 && N != 256 && N != 384 && N != 512)
    return ko::fail(KO_ERR_UNSUPPORTED, std::string(who) + ": N must be 128, 192, 256, 384 or 512");
  if (act != KO_ACT_NONE && act != KO_ACT_SILU)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": act must be KO_ACT_NONE or KO_ACT_SILU");
  if (!gamma || !beta || !(eps >= 0.0f) || !ko::aligned16(gamma) || !ko::aligned16(beta))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": gamma, beta required and 16-byte aligned; eps >= 0");
  if (y == x) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": y must not alias x");
  if ((ldx != 0 && (ldx < C || ldx % 4 != 0 || ldx > INT32_MAX)) ||
      (ldy != 0 && (ldy < N || ldy % 4 != 0 || ldy > INT32_MAX)))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": ldx / ldy must be 0 or multiples of 4 >= C / N");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool split = K > KO_SPLIT_MIN_K;
  const int bn = N == 384 ? 192 : N == 512 ? 256 : static_cast<int>(N);
  const int h = static_cast<int>(H), w = static_cast<int>(W), c = static_cast<int>(C);
#define KO_CONV_CASE(BNV)                                                                                        \
  if (bn == BNV)                                                                                                \
    return split ? launch_gemm_ln<BNV, true>(x, w_packed, bias, nullptr, nullptr, gamma, beta, eps, M, K, N, act, \
                                             nullptr, y, dev_status, s, h, w, c, ldx, ldy)                        \
                 : launch_gemm_ln<BNV, false>(x, w_packed, bias, nullptr, nullptr, gamma, beta, eps, M, K, N, act,\
                                              nullptr, y, dev_status, s, h, w, c, ldx, ldy);
  KO_CONV_CASE(128)
  KO_CONV_CASE(192)
  KO_CONV_CASE(256)
#undef KO_CONV_CASE
  return ko::fail(KO_ERR_UNSUPPORTED, std::string(who) + ": no tile for this N");
}

extern "C" int ko_linear_gelu_f32(const float* x, const float* w, const float* bias, int64_t M, int64_t K,
                                  int64_t N, float* out, void* workspace, int64_t workspace_bytes, int* dev_status,
                                  ko_stream_t stream) {
  int st = validate_linear(x, w, bias, M, K, N, out, "ko_linear_gelu_f32");
  if (st || M == 0) return st;
  if (!workspace || !ko::aligned16(workspace) || workspace_bytes < ko_linear_workspace_bytes(K, N))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_linear_gelu_f32: workspace missing, unaligned or too small");
  const ko::DeviceInfo* info = nullptr;
  st = ko::device_or_fail(&info, "ko_linear_gelu_f32");
  if (st) return st;
  float* packed = static_cast<float*>(workspace);
  st = ko_pack_weight_tf32x3(w, K, N, packed, stream);
  if (st) return st;
  return ko_linear_f32_packed(x, packed, bias, M, K, N, KO_ACT_GELU, out, dev_status, stream);
}

// ---------------------------------------------------------------------------------------------------------
// ko_linear_gelu_f32_noalloc: ko_linear_gelu_f32 with its scratch in library-owned static device memory.
//
// For callers that cannot allocate device memory themselves at run time (they cannot provide the workspace
// ko_linear_gelu_f32 asks for): applications whose allocator reserves all GPU memory up front and forbids
// libraries to allocate behind its back, per-frame real-time paths where cudaMalloc/cudaFree may synchronise
// the whole device and stall other streams, and plugin hosts that hand a plugin only its input and output
// buffers. The scratch — the tf32 hi/lo split of the weight, 2*K*N floats — lives in the file-scope array
// below instead, so this entry point never calls cudaMalloc, cudaFree or any allocating routine.
//
// Limits and sharing rules:
//   * K*N <= KO_NOALLOC_MAX_WEIGHT_ELEMS (2^20 elements; the array is 8 MiB and every GPU that loads this
//     library holds it until the process exits). Larger weights are rejected with KO_ERR_INVALID_ARGUMENT.
//   * Every call shares the one array per device. Calls that overlap on the GPU (different streams, or other
//     threads, without ordering between them) race on it and may produce wrong results: order them on one
//     stream or with events.
//   * Each call first rewrites the 2*K*N floats it uses, and the GEMM's tensor maps never read past them, so no
//     contents need clearing between calls (what the previous call left is overwritten before it is read).
//   * The first call on each device looks up the array's device address (cudaGetSymbolAddress, once per device,
//     with that device current); make that first call before any stream capture on that device.
// ---------------------------------------------------------------------------------------------------------
#include <mutex>
#include <vector>

namespace {

static __device__ __align__(256) float g_noalloc_wsplit[2 * KO_NOALLOC_MAX_WEIGHT_ELEMS];

// Device address of g_noalloc_wsplit on the current device (looked up once per device). The symbol's name in
// host code is only a host-side handle, never a device address, so it is never passed to a kernel itself.
int noalloc_scratch(float** out) {
  static std::mutex mu;
  static std::vector<float*> addr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ko::fail(static_cast<int>(e), "ko_linear_gelu_f32_noalloc: cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(addr.size()) <= dev) addr.resize(dev + 1, nullptr);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_wsplit);
    if (e != cudaSuccess || p == nullptr)
      return ko::fail(static_cast<int>(e ? e : cudaErrorInvalidSymbol),
                      std::string("ko_linear_gelu_f32_noalloc: cudaGetSymbolAddress failed: ") +
                          cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return KO_OK;
}

}  // namespace

extern "C" int ko_linear_gelu_f32_noalloc(const float* x, const float* w, const float* bias, int64_t M, int64_t K,
                                          int64_t N, float* out, int* dev_status, ko_stream_t stream) {
  int st = validate_linear(x, w, bias, M, K, N, out, "ko_linear_gelu_f32_noalloc");
  if (st || M == 0) return st;
  if (K * N > KO_NOALLOC_MAX_WEIGHT_ELEMS)
    return ko::fail(KO_ERR_INVALID_ARGUMENT,
                    "ko_linear_gelu_f32_noalloc: K*N = " + std::to_string(K * N) +
                        " exceeds the static scratch of KO_NOALLOC_MAX_WEIGHT_ELEMS = " +
                        std::to_string(static_cast<long long>(KO_NOALLOC_MAX_WEIGHT_ELEMS)) +
                        " weight elements; use ko_linear_gelu_f32 with a workspace instead");
  const ko::DeviceInfo* info = nullptr;
  st = ko::device_or_fail(&info, "ko_linear_gelu_f32_noalloc");
  if (st) return st;
  float* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  st = ko_pack_weight_tf32x3(w, K, N, scratch, stream);
  if (st) return st;
  return ko_linear_f32_packed(x, scratch, bias, M, K, N, KO_ACT_GELU, out, dev_status, stream);
}
