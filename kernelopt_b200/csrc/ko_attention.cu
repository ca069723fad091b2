// Multi-head scaled-dot-product attention in fp32 grade on the B200 5th-generation tensor cores (tcgen05,
// kind::tf32, 3xTF32), flash style: the L x L score matrix never leaves the SM.
//
//   o[b, i, h, :] = sum_j softmax_j(scale * q[b, i, h, :] . k[b, j, h, :]) v[b, j, h, :]
//
// Semantics: the reference's attention calls, mx.fast.scaled_dot_product_attention on head-major q/k/v in the
// ViT backbone (fast_rfdetr/model.py:107-110 and 119-120, windowed and global layers) and in the decoder's
// self-attention (self_attn, model.py:232-239, 8 heads of 32), computed in fp32 there. No mask, no dropout.
//
// Precision: every operand is split v = hi + lo and the tensor cores accumulate hi*hi + hi*lo + lo*hi in fp32
// (Ootomo & Yokota's error-compensated 3xTF32). q and k, whose products the exponential amplifies, use
// hi = tf32_rn(v); p and v use hi = v itself, which the tensor core reads truncated to tf32, and lo = the exact
// remainder below that truncation (two operations per element instead of three; error below 2^-20 per term). The
// softmax runs in fp32 registers with the running maximum / running sum of the online (flash) formulation; each
// key block's P.V product lands in a fresh tensor-memory accumulator and is added into the fp32 output row in
// registers, so the long sum over keys is a plain fp32 register sum, not a tensor-core accumulation.
//
// Kernel structure: pairs of CTAs (clusters of two on one GPU), as many as the GPU holds at once, 13 warps each;
// each pair loops over work items (two 128-query tiles, head, batch item), the key blocks of all its items forming
// one pipeline: the next item's q tile loads while the current item's last blocks run, so a short sequence (a
// 401-token window: four key blocks) does not pay a whole CTA prologue per item. The pair runs the 5th-generation
// tensor cores of two SMs as one (tcgen05 cta_group::2): every MMA has M = 256, rows 0-127 being the leader's
// (rank 0) query tile and 128-255 the peer's, each CTA holding its own A rows and HALF of B at the same
// shared-memory offset and receiving its 128 rows of the product in its own tensor memory. So each SM loads,
// splits and stores only half of each k / v tile, and its tensor core reads only half of each B operand; and the
// halves fit twice in shared memory, so the loaders write block j + 1 while block j's MMAs read block j (with
// one buffer, each block's k and v writes waited for the previous block's MMAs).
//   warp 0      allocates the pair's tensor memory; in the leader, one lane issues the MMAs of both CTAs:
//                 S  = Q K_j^T      (M 256, N = 128 keys, K = head dim;  A, B in shared memory)
//                 O_j = P_j V_j     (M 256, N = head dim, K = 128 keys; A = P in tensor memory, B in shared)
//   warps 1-4   softmax + output: one thread per query row. Reads S from tensor memory, updates the row's running
//               max / sum, writes P (hi and lo) back into tensor memory for the P.V MMA, then adds O_j into the
//               output row it keeps in registers. At the end divides by the sum and stores the row.
//   warps 5-12  loaders: per item, warps 9-12 load the q tile by TMA once the previous item's last S MMA has read
//               the q buffer, and split it in place; key blocks stream from global memory (128-bit loads; warps
//               5-8 stream this CTA's k rows, 9-12 its v columns, each holding the next half tile, of the same
//               item or the next, in registers), split into hi / lo and written into one of two shared-memory buffers
//               with 128-bit stores: k in the S MMA's 128-byte-swizzled K-major layout; v (head dim 64) as it is,
//               keys x this CTA's 32 head-dim columns, which the P.V MMA reads as an MN-major B operand (head dim
//               32 leaves a CTA 16 columns, less than one MN-major row: that v is written transposed, head dim x
//               keys, the K-major form).
// A query tile count that is odd gets one more tile of padding rows (zero queries, never stored).
// Tensor memory (512 columns per CTA): two S / P_hi buffers [0,256), P_lo [256,384), two O_j buffers of HD columns
// from 384. With two S buffers the tensor cores compute S_{j+1} while the softmax warps work on block j, and
// P_j.V_j issues its P_lo products first and then frees the one P_lo buffer, so the softmax warps write P_{j+1}
// while the P_hi products of block j run (the softmax of one block overlaps the tensor-core work of the previous).
// Barriers that the leader's MMA lane waits on count arrivals from both CTAs (the peer arrives through the
// cluster-mapped address of the leader's barrier, after the same proxy / tensor-memory fences as a local arrival);
// each MMA completion is committed to the same barrier in both CTAs. Every wait on an mbarrier is bounded (2 s); on
// timeout the CTA stops, drains its MMAs, frees tensor memory and reports KO_ERR_DEVICE_TIMEOUT through dev_status.
#include <algorithm>
#include <climits>
#include <string>

#include "ko_common.cuh"

namespace {

using namespace kodev;

constexpr int BQ = 128;            // query rows per CTA (half of the pair's MMA M)
constexpr int BKEY = 128;          // keys per block (MMA N of S, K of P.V)
constexpr int KHALF = BKEY / 2;    // k rows of a block held by one CTA of the pair (at most)
constexpr int kLoadWarp0 = 5;
constexpr int kLoadThreads = 256;
constexpr int kThreads = 13 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;      // two S / P_hi buffers of 128 columns
constexpr uint32_t kColPlo = 256;  // P_lo, 128 columns
constexpr uint32_t kColO = 384;    // two O_j buffers of HD columns

struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  int64_t q_bstride, k_bstride, v_bstride, o_bstride;  // elements between consecutive batch items
  int q_row, k_row, v_row, o_row;                      // elements between consecutive tokens
  int L, n_kblocks;
  int heads, pairs;              // query-tile pairs per sequence (an odd tile count gets a padding tile)
  int total_items, n_clusters;   // work items (pair, head, batch item) and the CTA pairs that share them
  float scale_log2;  // softmax scale * log2(e): exponentials are taken as exp2
  int* dev_status;
};

template <int HD>
struct AttnCfg {
  static constexpr int kKB = HD / 32;                          // 128-byte k-blocks of a q / k row
  static constexpr uint32_t kQBytes = BQ * HD * 4;             // one of Q_hi / Q_lo
  static constexpr uint32_t kKBytes = KHALF * HD * 4;          // one of K_hi / K_lo of this CTA's k rows
  static constexpr uint32_t kVBytes = (HD / 2) * BKEY * 4;     // one of Vt_hi / Vt_lo of this CTA's v columns
  static constexpr uint32_t kKBufBytes = 2 * kKBytes;          // a k buffer: [K_hi][K_lo]
  static constexpr uint32_t kVBufBytes = 2 * kVBytes;          // a v buffer: [Vt_hi][Vt_lo]
  static constexpr uint32_t kOffQlo = kQBytes;
  static constexpr uint32_t kOffK = 2 * kQBytes;               // two k buffers (block j in buffer j & 1)
  static constexpr uint32_t kOffV = kOffK + 2 * kKBufBytes;    // two v buffers
  static constexpr uint32_t kOffBars = kOffV + 2 * kVBufBytes;
  // At least 120 KB even where the tiles need less (head dim 32), so that one CTA per SM holds all 512 tensor-
  // memory columns and no second CTA waits in tcgen05.alloc.
  static constexpr uint32_t kOffRowPtr = kOffBars + 256;  // [BQ] output-row pointers of the softmax threads
  static constexpr size_t kSmemNeed = 1024 + kOffRowPtr + BQ * 8;
  static constexpr size_t kSmemBytes = kSmemNeed > 120 * 1024 ? kSmemNeed : 120 * 1024;
  static_assert(HD == 32 || HD == 64, "head dim 32 or 64");
};

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a K-major tile of 128-byte rows, 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// v = hi + lo with hi = tf32_rn(v). lo = v - hi is exact in fp32 and is left unrounded: the tensor core reads a
// tf32 operand from its top 19 bits, so lo enters the product truncated to tf32, an error below 2^-21 |v|
// (2^-22 with lo rounded first), which saves the second rounding's two integer operations.
__device__ __forceinline__ void split_tf32(float v, float& hi, float& lo) {
  hi = __uint_as_float(f32_to_tf32_rna_int(v));
  lo = v - hi;
}

// 32 lanes x 16 consecutive 32-bit columns, load and store.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait_regs16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// mbarrier wait whose result is the same in every lane of the warp (the warp then runs .sync.aligned tcgen05
// operations together, or leaves its loop together).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Shared-memory descriptor of an MN-major tf32 operand tile: 128-byte rows of the M / N dimension (32 values), 4-row
// atoms along K 512 bytes apart, the 32-byte chunks of a row permuted by chunk ^ (row & 3) (for 32-bit types the
// MN-major form takes this 128-byte swizzle with 32-byte atoms, layout type 1), atoms on 512-byte boundaries.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128_32b(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);         // start address
  // leading byte offset: the next 32 columns. A CTA's half has one 32-column group, so it is never used, but it
  // must be a real offset: 16 bytes here made the MMA fault with a misaligned address.
  d |= static_cast<uint64_t>((16384u >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;   // stride byte offset: next 4 rows of K
  d |= static_cast<uint64_t>(1u) << 46;                       // descriptor version (sm_100)
  d |= static_cast<uint64_t>(1u) << 61;                       // layout: 128-byte swizzle, 32-byte atoms
  return d;
}

// tcgen05 of a CTA pair (cta_group::2): every tcgen05 operation of the kernel names the pair. The allocation is made
// by warp 0 of both CTAs with the same destination slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A B over the pair, A and B from shared memory (elected lane of the calling warp).
__device__ __forceinline__ void mma_pair_tf32_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same with A in tensor memory (each CTA's 128 lanes).
__device__ __forceinline__ void mma_pair_tf32_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                   uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` in both CTAs of the pair when every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b16 mask;\n\tmov.b16 mask, 3;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], mask;\n\t}"
      ::"r"(smem_addr(bar))
      : "memory");
}

// The part of v below its tf32 truncation: v - (v with the low 13 mantissa bits cleared), exact in fp32. P is kept
// as v in the P_hi slot (the tensor core reads a tf32 operand from the top 19 bits of the word, i.e. truncates)
// and this tail in P_lo, so P = P_hi + P_lo exactly before the MMA truncates P_lo (an error below 2^-20 P).
__device__ __forceinline__ float tf32_tail(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x by the MUFU (ex2.approx, relative error below 2^-22 over the range used here: x <= 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) attention_tf32x3_kernel(const __grid_constant__ CUtensorMap map_q,
                                                                        const AttnArgs a) {
  using C = AttnCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  // Barriers the leader's MMA warp waits on collect arrivals from both CTAs of the pair; the MMA commits arrive on
  // the same barrier in both CTAs (multicast). Block phases run over the pair's whole sequence of key blocks
  // (g = item * nkb + j), so the pipeline continues from one work item into the next.
  uint64_t* q_ready = bars + 0;   // q tile split            (4 v-loader warps x 2 CTAs, leader)
  uint64_t* k_full = bars + 1;    // k half tile written, x2 (4 k-loader warps x 2 CTAs, leader)
  uint64_t* v_full = bars + 3;    // v half tile written, x2 (4 v-loader warps x 2 CTAs, leader)
  uint64_t* s_full = bars + 5;    // S_g complete, x2        (1 commit, both CTAs)
  uint64_t* p_full = bars + 7;    // P_g written             (4 softmax warps x 2 CTAs, leader)
  uint64_t* o_full = bars + 8;    // O_g complete, x2        (1 commit, both CTAs)
  uint64_t* mma_done = bars + 12;  // every MMA complete      (1 commit, both CTAs)
  uint64_t* plo_free = bars + 13;  // P_g.V_g's P_lo products done (1 commit, both CTAs)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  uint64_t* q_tma = bars + 15;     // q tile landed (fp32)     (1 arrival + tx bytes)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the pair's MMAs
  const int nkb = a.n_kblocks;
  // Work items (query-tile pair, head, batch item), the pair index fastest so that concurrent pairs share k / v
  // in L2; this pair takes items cluster, cluster + n_clusters, ...
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int n_items = cluster < a.total_items ? (a.total_items - cluster + a.n_clusters - 1) / a.n_clusters : 0;
  const int n_blocks = n_items * nkb;  // key blocks of all this pair's items, in order
  struct Item {
    int b, h, q0;
  };
  auto item_of = [&](int k) -> Item {
    const int it = cluster + k * a.n_clusters;
    const int pr = it % a.pairs, rest = it / a.pairs;
    return Item{rest / a.heads, rest % a.heads, (2 * pr + static_cast<int>(rank)) * BQ};
  };
  // keys of block j of an item, the S MMA's N (keys rounded up to 16) and this CTA's share of the block's k rows
  // (N / 2, starting at rank * N / 2)
  auto keys_of = [&](int j) { return min(BKEY, a.L - j * BKEY); };
  auto n_of = [&](int j) { return (keys_of(j) + 15) & ~15; };
  // Arrive on the leader's copy of a barrier (this CTA's own when it is the leader): the leader's barrier area is
  // mapped once, the barrier's offset within it is a constant. The arrival has the default (CTA-scope release)
  // semantics; a cluster-scope release costs a cluster-wide memory barrier per arrival, which stalled the
  // softmax and loader warps (10 % of the kernel's time).
  const uint32_t leader_bars = cluster_map(smem_addr(bars), 0);
  auto arrive_leader = [&](uint64_t* bar) {
    const uint32_t addr = leader_bars + static_cast<uint32_t>(reinterpret_cast<uint8_t*>(bar) -
                                                               reinterpret_cast<uint8_t*>(bars));
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
  };

  if (threadIdx.x == 0) {
    mbar_init(q_ready, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 8);
      mbar_init(&v_full[i], 8);
      mbar_init(&s_full[i], 1);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(p_full, 8);
    mbar_init(mma_done, 1);
    mbar_init(plo_free, 1);
    mbar_init(q_tma, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any arrival from the peer
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (rank == 0 && n_blocks > 0) {
      // ---------------- MMA issuer (leader) ----------------
      // Order on the tensor pipes of the pair: S_0, then per block g: S_{g+1} (into the other S buffer,
      // overlapping softmax_g), P_g.V_g. S_{g+1} reuses the buffer of P_{g-1}, so it waits for P_{g-1}.V_{g-1}.
      // Each MMA has M = 256: rows 0-127 are the leader's query tile, 128-255 the peer's, each CTA holding its A
      // rows (q, or P in its tensor memory) and half of B (k rows, or v columns) at the same shared-memory offset,
      // and receiving its 128 rows of the product in its own tensor memory. The first S of an item waits for its
      // q tile, which the loaders write once the previous item's last S is complete.
      // The whole warp runs this loop with the same values in every lane; one elected lane issues each MMA.
      const uint32_t sb = smem_addr(smem);
      // head dim 64: each CTA's v half (32 columns) is one 128-byte MN-major column group; bit 16 = B MN-major
      constexpr bool kVMN = HD == 64;
      constexpr uint32_t idesc_o = idesc_tf32(2 * BQ, HD) | (kVMN ? (1u << 16) : 0u);
      const uint64_t dq_hi = smem_desc_k_sw128(sb), dq_lo = smem_desc_k_sw128(sb + C::kOffQlo);
      auto issue_s = [&](int g) {  // S_g = Q K_g^T into S buffer g & 1
        const int j = g % nkb;
        const uint32_t d = tmem + kColS + static_cast<uint32_t>(g & 1) * BKEY;
        const uint32_t idesc_s = idesc_tf32(2 * BQ, n_of(j));
        const uint32_t kb0 = sb + C::kOffK + static_cast<uint32_t>(g & 1) * C::kKBufBytes;
        const uint64_t dk_hi = smem_desc_k_sw128(kb0), dk_lo = smem_desc_k_sw128(kb0 + C::kKBytes);
#pragma unroll
        for (int s = 0; s < C::kKB * 4; ++s) {  // 8-wide k-steps over the head dimension
          const uint64_t qoff = static_cast<uint64_t>(((s >> 2) * (BQ * 128) + (s & 3) * 32) >> 4);
          const uint64_t koff = static_cast<uint64_t>(((s >> 2) * (KHALF * 128) + (s & 3) * 32) >> 4);
          mma_pair_tf32_w(d, dq_lo + qoff, dk_hi + koff, idesc_s, s == 0 ? 0u : 1u);
          mma_pair_tf32_w(d, dq_hi + qoff, dk_lo + koff, idesc_s, 1u);
          mma_pair_tf32_w(d, dq_hi + qoff, dk_hi + koff, idesc_s, 1u);
        }
        mma_commit_pair_w(&s_full[g & 1]);  // the loaders wait on it too (S_g done = k buffer g & 1 free)
      };
      // block g may issue its S once its item's q tile is split and its k half tile written
      auto s_ready = [&](int g) -> bool {
        if (g % nkb == 0 && !warp_wait(q_ready, static_cast<uint32_t>(g / nkb) & 1u, abort_flag)) return false;
        return warp_wait(&k_full[g & 1], static_cast<uint32_t>(g >> 1) & 1u, abort_flag);
      };
      bool ok = s_ready(0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      // S_{g+1} (buffer (g + 1) & 1 held P_{g-1}: P_{g-1}.V_{g-1} must be complete)
      auto next_s = [&](int g) -> bool {
        if (!s_ready(g + 1)) return false;
        if (g >= 1 && !warp_wait(&o_full[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, abort_flag))
          return false;
        tc_fence_after();
        issue_s(g + 1);
        return true;
      };
      for (int g = 0; g < n_blocks && ok; ++g) {
        if (g + 1 < n_blocks && !next_s(g)) break;
        // O_g = P_g V_g into O buffer g & 1, once P_g is written and V_g landed. The buffer held O_{g-2}, which
        // every softmax warp read (add_block(g - 2)) before it wrote P_g: p_full covers it.
        if (!warp_wait(p_full, static_cast<uint32_t>(g) & 1u, abort_flag) ||
            !warp_wait(&v_full[g & 1], static_cast<uint32_t>(g >> 1) & 1u, abort_flag))
          break;
        tc_fence_after();
        const uint32_t d = tmem + kColO + static_cast<uint32_t>(g & 1) * HD;
        const uint32_t p_hi = tmem + kColS + static_cast<uint32_t>(g & 1) * BKEY;
        const uint32_t vb0 = sb + C::kOffV + static_cast<uint32_t>(g & 1) * C::kVBufBytes;
        const uint64_t dv_hi = kVMN ? smem_desc_mn_sw128_32b(vb0) : smem_desc_k_sw128(vb0);
        const uint64_t dv_lo = kVMN ? smem_desc_mn_sw128_32b(vb0 + C::kVBytes) : smem_desc_k_sw128(vb0 + C::kVBytes);
        // k-step kk (8 keys): MN-major, 8 rows of 128 bytes; K-major, 32 bytes within a 32-key row block
        auto voff = [&](int kk) {
          return static_cast<uint64_t>(kVMN ? kk * 64 : ((kk >> 2) * (HD / 2 * 128) + (kk & 3) * 32) >> 4);
        };
        const int ksteps = (keys_of(g % nkb) + 7) >> 3;
        // The P_lo products first, then a commit that hands the P_lo columns back to the softmax warps: they
        // write P_{g+1} while the P_hi products of this block (two thirds of its MMAs) still run. A full block's
        // MMAs are issued from fully unrolled code (a rolled loop's address arithmetic would make the issue, not
        // the pipe, the limit).
        if (ksteps == BKEY / 8) {
#pragma unroll
          for (int kk = 0; kk < BKEY / 8; ++kk) {  // 8 keys per k-step
            mma_pair_tf32_ts_w(d, tmem + kColPlo + 8 * kk, dv_hi + voff(kk), idesc_o, kk == 0 ? 0u : 1u);
          }
          mma_commit_pair_w(plo_free);
#pragma unroll
          for (int kk = 0; kk < BKEY / 8; ++kk) {
            mma_pair_tf32_ts_w(d, p_hi + 8 * kk, dv_lo + voff(kk), idesc_o, 1u);
            mma_pair_tf32_ts_w(d, p_hi + 8 * kk, dv_hi + voff(kk), idesc_o, 1u);
          }
        } else {  // a short last block
#pragma unroll 1
          for (int kk = 0; kk < ksteps; ++kk) {
            mma_pair_tf32_ts_w(d, tmem + kColPlo + 8 * kk, dv_hi + voff(kk), idesc_o, kk == 0 ? 0u : 1u);
          }
          mma_commit_pair_w(plo_free);
#pragma unroll 1
          for (int kk = 0; kk < ksteps; ++kk) {
            mma_pair_tf32_ts_w(d, p_hi + 8 * kk, dv_lo + voff(kk), idesc_o, 1u);
            mma_pair_tf32_ts_w(d, p_hi + 8 * kk, dv_hi + voff(kk), idesc_o, 1u);
          }
        }
        // One commit per event: the v loaders wait on o_full as well (P_g.V_g done = v buffer g & 1 free).
        mma_commit_pair_w(&o_full[g & 1]);
      }
    }
    // Drain: every MMA the leader issued completes before either CTA releases its tensor memory.
    if (rank == 0) mma_commit_pair_w(mma_done);
    volatile int never = 0;
    if (!warp_wait(mma_done, 0, &never)) *abort_flag = 1;
  } else if (warp < kLoadWarp0) {
    // ---------------- softmax + output, one thread per query row ----------------
    // Block g (key block j of item g / nkb), two passes over S_g in tensor memory: the first finds the row
    // maximum, which sets the block's offset m = max(m, block maximum) (online softmax, P <= 1); once
    // P_{g-1}.V_{g-1}'s P_lo products are done (the P_lo columns are free) the second turns each 16-key chunk
    // into P = exp2(S * c - m), written as P itself and its tf32 tail. The max pass overlaps that wait. Then,
    // once all of P_{g-1}.V_{g-1} is complete, o = o * alpha + that block's product. An item's first block starts
    // from m = -inf, so its alpha is 0 and the fold of its first product replaces o; the previous item's row is
    // finished (its last fold, the division by its sum and the store) just before that.
    const int quad = warp & 3;  // tensor-memory lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    auto add_block = [&](int gb, float alpha) -> bool {  // o = o * alpha + O_gb
      if (!warp_wait(&o_full[gb & 1], static_cast<uint32_t>(gb >> 1) & 1u, abort_flag)) return false;
      tc_fence_after();
      const uint32_t ob = trow + kColO + static_cast<uint32_t>(gb & 1) * HD;
#pragma unroll
      for (int c = 0; c < HD / 16; ++c) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(ob + 16 * c, r);
        tmem_ld_wait_regs16(r);
#pragma unroll
        for (int e = 0; e < 16; ++e) o[16 * c + e] = fmaf(o[16 * c + e], alpha, __uint_as_float(r[e]));
      }
      return true;
    };
    // This thread's output row of item k (null for a padding row), and the store of the finished row.
    auto row_ptr = [&](int k) -> float4* {
      const Item itm = item_of(k);
      const int qi = itm.q0 + row;
      if (qi >= a.L) return nullptr;
      return reinterpret_cast<float4*>(a.o + static_cast<int64_t>(itm.b) * a.o_bstride +
                                       static_cast<int64_t>(qi) * a.o_row + itm.h * HD);
    };
    auto store_row = [&](float4* dst, float l_row) {
      if (dst == nullptr) return;
      const float inv = 1.0f / l_row;
#pragma unroll
      for (int d = 0; d < HD / 4; ++d)
        dst[d] = make_float4(o[4 * d] * inv, o[4 * d + 1] * inv, o[4 * d + 2] * inv, o[4 * d + 3] * inv);
    };
    // the current item's row pointer waits in shared memory (in registers it pushed the loop over its budget)
    float4** orow = reinterpret_cast<float4**>(smem + C::kOffRowPtr) + row;
    *orow = n_blocks > 0 ? row_ptr(0) : nullptr;
    for (int g = 0; g < n_blocks; ++g) {
      const int j = g % nkb;
      if (j == 0) m = -INFINITY;  // a new item: its first block's alpha is 0, which also restarts the sum
      if (!warp_wait(&s_full[g & 1], static_cast<uint32_t>(g >> 1) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = trow + kColS + static_cast<uint32_t>(g & 1) * BKEY;
      const uint32_t plrow = trow + kColPlo;
      const int valid = keys_of(j);
      const int chunks = (valid + 15) >> 4;  // 16-column chunks that hold keys of this block
      // pass 1: the block's row maximum
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < chunks; ++c) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(srow + 16 * c, r);
        tmem_ld_wait_regs16(r);
        const int nv = valid - 16 * c;  // keys of this chunk (>= 16 except in a short last block)
        if (nv < 16) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e >= nv) r[e] = __float_as_uint(-INFINITY);
        }
        const float* f = reinterpret_cast<const float*>(r);
        const float m0 = fmax3(f[0], f[1], f[2]), m1 = fmax3(f[3], f[4], f[5]), m2 = fmax3(f[6], f[7], f[8]);
        const float m3 = fmax3(f[9], f[10], f[11]), m4 = fmax3(f[12], f[13], f[14]);
        mx = fmax3(mx, fmax3(m0, m1, m2), fmax3(m3, m4, f[15]));
      }
      const float mb = fmaxf(m, mx * a.scale_log2);  // offset of this block's P
      if (g >= 1 && !warp_wait(plo_free, static_cast<uint32_t>(g - 1) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // pass 2: P and its tail; two partial sums shorten the dependent chain of additions
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll 1
      for (int c = 0; c < chunks; ++c) {
        uint32_t r[16], lo[16];
        tmem_ld_32x32b_x16(srow + 16 * c, r);
        tmem_ld_wait_regs16(r);
        const int nv = valid - 16 * c;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float p = fast_exp2(fmaf(__uint_as_float(r[e]), a.scale_log2, -mb));
          if (e >= nv) p = 0.f;  // keys past the end of a short last block
          if (e & 1) ls1 += p; else ls0 += p;
          r[e] = __float_as_uint(p);  // read by the MMA as its top 19 bits: P_hi = P truncated to tf32
          lo[e] = __float_as_uint(tf32_tail(p));
        }
        tmem_st_32x32b_x16(srow + 16 * c, r);
        tmem_st_32x32b_x16(plrow + 16 * c, lo);
      }
      const float ls = ls0 + ls1;
      tmem_st_wait();
      const float alpha = fast_exp2(m - mb);  // 0 for an item's first block (m = -inf)
      const float l_done = l;                 // the previous item's sum when j == 0 (stored below)
      l = l * alpha + ls;
      m = mb;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(p_full);
      if (g >= 1) {
        if (!add_block(g - 1, alpha_prev)) {
          ok = false;
          break;
        }
        if (j == 0) {  // block g - 1 was the previous item's last: finish its row, start the next from zero
          store_row(*orow, l_done);
          *orow = row_ptr(g / nkb);
#pragma unroll
          for (int d = 0; d < HD; ++d) o[d] = 0.f;
        }
      }
      alpha_prev = alpha;
    }
    if (ok && n_blocks > 0 && add_block(n_blocks - 1, alpha_prev)) store_row(*orow, l);
  } else {
    // ---------------- loaders ----------------
    // Per item the v group (warps 9-12) loads the q tile by TMA, once the previous item's last S MMA has read the
    // q buffer, and splits it in place. Warps 5-8 stream this CTA's k halves (its N / 2 keys of each block) and
    // warps 9-12 its v halves (all keys of a block, head-dim columns [rank * HD / 2, (rank + 1) * HD / 2)), into
    // alternating buffers, each group holding its next half tile (of the same item or the next) in registers
    // while the current one is written.
    const int t = threadIdx.x - kLoadWarp0 * 32;  // 0..255
    constexpr int Q4 = HD / 4;                   // float4 per q / k row
    constexpr int kGroup = kLoadThreads / 2;     // 128 threads per group
    constexpr int kTileChunks = KHALF * HD / 4 / kGroup;  // float4 per thread of a half tile (k or v)
    const int g0 = t & (kGroup - 1);
    float4 reg[kTileChunks];
    if (t < kGroup) {
      // k halves: row-major chunks (a warp reads whole rows), stored K-major with the 128-byte swizzle
      auto load = [&](int g) {
        const Item itm = item_of(g / nkb);
        const int j = g % nkb;
        const float* kbp = a.k + static_cast<int64_t>(itm.b) * a.k_bstride + itm.h * HD;
        const int half = n_of(j) / 2, r0 = j * BKEY + static_cast<int>(rank) * half;
#pragma unroll
        for (int i = 0; i < kTileChunks; ++i) {
          const int idx = i * kGroup + g0, r = idx / Q4, kr = r0 + r, kc = idx % Q4;
          reg[i] = r < half && kr < a.L
                       ? __ldg(reinterpret_cast<const float4*>(kbp + static_cast<int64_t>(kr) * a.k_row) + kc)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      };
      if (n_blocks > 0) load(0);
      for (int g = 0; g < n_blocks; ++g) {
        // k buffer g & 1 held block g - 2: S_{g-2} must be complete
        if (g >= 2 && !mbar_wait(&s_full[g & 1], static_cast<uint32_t>((g - 2) >> 1) & 1u, abort_flag)) break;
        const uint32_t kbuf = C::kOffK + static_cast<uint32_t>(g & 1) * C::kKBufBytes;
#pragma unroll
        for (int i = 0; i < kTileChunks; ++i) {
          const int idx = i * kGroup + g0, r = idx / Q4, c = idx % Q4;
          const uint32_t off = (c >> 3) * (KHALF * 128) + sw128(r, c & 7);
          float4 hi, lo;
          split_tf32(reg[i].x, hi.x, lo.x);
          split_tf32(reg[i].y, hi.y, lo.y);
          split_tf32(reg[i].z, hi.z, lo.z);
          split_tf32(reg[i].w, hi.w, lo.w);
          *reinterpret_cast<float4*>(smem + kbuf + off) = hi;
          *reinterpret_cast<float4*>(smem + kbuf + C::kKBytes + off) = lo;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_leader(&k_full[g & 1]);
        if (g + 1 < n_blocks) load(g + 1);
      }
    } else {
      // v halves: a thread reads one key's HD / 2 columns of this CTA's half (8 or 4 float4)
      auto load = [&](int g) {
        const Item itm = item_of(g / nkb);
        const int vr = (g % nkb) * BKEY + g0;
        const float* vbp =
            a.v + static_cast<int64_t>(itm.b) * a.v_bstride + itm.h * HD + static_cast<int>(rank) * (HD / 2);
#pragma unroll
        for (int i = 0; i < kTileChunks; ++i)
          reg[i] = vr < a.L ? __ldg(reinterpret_cast<const float4*>(vbp + static_cast<int64_t>(vr) * a.v_row) + i)
                            : make_float4(0.f, 0.f, 0.f, 0.f);  // keys past the end: P is 0 there, v must be finite
      };
      if (n_blocks > 0) load(0);
      bool vok = true;
      for (int g = 0; g < n_blocks && vok; ++g) {
        if (g % nkb == 0) {
          // q of item g / nkb: the previous item's last S (block g - 1) has read the q buffer
          const int k = g / nkb;
          if (g >= 1 && !mbar_wait(&s_full[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, abort_flag)) break;
          if (g0 == 0) {
            const Item itm = item_of(k);
            const int bq = a.q_bstride ? itm.b : 0;
            mbar_arrive_expect_tx(q_tma, C::kQBytes);
#pragma unroll
            for (int kb = 0; kb < C::kKB; ++kb)
              tma_load_3d(&map_q, q_tma, smem + kb * (BQ * 128), itm.h * HD + kb * 32, itm.q0, bq);
          }
          if (!mbar_wait(q_tma, static_cast<uint32_t>(k) & 1u, abort_flag)) break;
          // hi in place, lo at the same offset in the lo buffer (elementwise: any cover of the tile works)
          for (int i = g0; i < static_cast<int>(C::kQBytes / 16); i += kGroup) {
            float4* src = reinterpret_cast<float4*>(smem) + i;
            const float4 v = *src;
            float4 hi, lo;
            split_tf32(v.x, hi.x, lo.x);
            split_tf32(v.y, hi.y, lo.y);
            split_tf32(v.z, hi.z, lo.z);
            split_tf32(v.w, hi.w, lo.w);
            *src = hi;
            reinterpret_cast<float4*>(smem + C::kOffQlo)[i] = lo;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) arrive_leader(q_ready);
        }
        // v buffer g & 1 held block g - 2: P_{g-2}.V_{g-2} must be complete
        if (g >= 2 && !mbar_wait(&o_full[g & 1], static_cast<uint32_t>((g - 2) >> 1) & 1u, abort_flag)) break;
        const uint32_t vbuf = C::kOffV + static_cast<uint32_t>(g & 1) * C::kVBufBytes;
        const int key = g0;
        if constexpr (HD == 64) {
          // as it is: row `key` of 128 bytes, its 16-byte chunk i at (i ^ ((key & 3) << 1)), 128-bit stores
#pragma unroll
          for (int i = 0; i < kTileChunks; ++i) {
            const uint32_t off = key * 128 + ((i ^ ((key & 3) << 1)) << 4);
            // v itself as hi (read truncated to tf32) and its tail as lo: P.V errors are not amplified
            const float4 lo = make_float4(tf32_tail(reg[i].x), tf32_tail(reg[i].y), tf32_tail(reg[i].z),
                                          tf32_tail(reg[i].w));
            *reinterpret_cast<float4*>(smem + vbuf + off) = reg[i];
            *reinterpret_cast<float4*>(smem + vbuf + C::kVBytes + off) = lo;
          }
        } else {
          // transposed (head dim x keys, K-major, 128-byte swizzle): every scalar store of a warp fills one
          // 128-byte row (32 consecutive keys of one head-dim column)
          const uint32_t base = (key >> 5) * (HD / 2 * 128) + ((key & 3) << 2);
#pragma unroll
          for (int i = 0; i < kTileChunks; ++i) {
            const float* src = reinterpret_cast<const float*>(&reg[i]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int d = 4 * i + e;  // head-dim column within this CTA's half
              const uint32_t off = base + sw128(d, (key & 31) >> 2);
              const float hi = src[e], lo = tf32_tail(src[e]);  // v itself as hi: P.V errors are not amplified
              *reinterpret_cast<float*>(smem + vbuf + off) = hi;
              *reinterpret_cast<float*>(smem + vbuf + C::kVBytes + off) = lo;
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_leader(&v_full[g & 1]);
        if (g + 1 < n_blocks) load(g + 1);
      }
    }
  }

  // Neither CTA leaves while the other may still arrive on its barriers or (the leader's MMAs) read its shared and
  // tensor memory: every MMA is complete (mma_done, waited by warp 0 of each CTA above) and every thread of the
  // pair is past its last arrival.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && a.dev_status) atomicExch(a.dev_status, KO_ERR_DEVICE_TIMEOUT);
}

}  // namespace

extern "C" int ko_attention_f32(const float* q, const float* k, const float* v, float* o, int64_t batch, int64_t L,
                                int64_t heads, int64_t head_dim, int64_t q_bstride, int64_t q_row,
                                int64_t k_bstride, int64_t k_row, int64_t v_bstride, int64_t v_row,
                                int64_t o_bstride, int64_t o_row, float scale, int* dev_status, ko_stream_t stream) {
  const char* who = "ko_attention_f32";
  if (head_dim != 32 && head_dim != 64)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": head_dim must be 32 or 64");
  if (batch < 0 || L < 0 || heads < 1 || batch > 65535 || heads > 65535 || L > (int64_t(1) << 30))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": bad batch / length / heads");
  if (batch == 0 || L == 0) return KO_OK;
  if (!q || !k || !v || !o) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  const int64_t strides[8] = {q_bstride, q_row, k_bstride, k_row, v_bstride, v_row, o_bstride, o_row};
  for (int64_t st : strides)
    if (st < 0 || st % 4 != 0 || st > INT32_MAX * int64_t(4))
      return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": strides must be non-negative multiples of 4");
  if (q_row > INT32_MAX || k_row > INT32_MAX || v_row > INT32_MAX || o_row > INT32_MAX)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": row stride too large");
  if (heads * head_dim > q_row || heads * head_dim > k_row || heads * head_dim > v_row || heads * head_dim > o_row)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": a row must hold heads * head_dim values");
  if (!ko::aligned16(q) || !ko::aligned16(k) || !ko::aligned16(v) || !ko::aligned16(o))
    return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": pointers must be 16-byte aligned");
  if (!(scale > 0.0f)) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": scale must be positive");
  AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.o = o;
  a.q_bstride = q_bstride;
  a.k_bstride = k_bstride;
  a.v_bstride = v_bstride;
  a.o_bstride = o_bstride;
  a.q_row = static_cast<int>(q_row);
  a.k_row = static_cast<int>(k_row);
  a.v_row = static_cast<int>(v_row);
  a.o_row = static_cast<int>(o_row);
  a.L = static_cast<int>(L);
  a.n_kblocks = static_cast<int>((L + BKEY - 1) / BKEY);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.dev_status = dev_status;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // q tiles by TMA: [batch][L][heads * head_dim] with the caller's strides, boxes of 32 columns x 128 rows; a
  // stride of 0 between batch items maps every item to plane 0
  CUtensorMap mq;
  const uint64_t width = static_cast<uint64_t>(heads * head_dim);
  int rc = ko::make_tmap_3d_f32(&mq, q, q_bstride ? batch : 1, L, width, q_row,
                                q_bstride ? q_bstride : q_row * L + 4, BQ, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                                "ko_attention_f32 q");
  if (rc) return rc;
  // Work items: query tiles in pairs (an odd count gets one tile of padding rows) x heads x batch items, spread
  // over as many CTA pairs (clusters of two) as the GPU holds at once; each pair loops over its items.
  const int64_t qtiles = (L + BQ - 1) / BQ;
  const int64_t pairs = (qtiles + 1) / 2, total = pairs * heads * batch;
  if (total > INT32_MAX) return ko::fail(KO_ERR_INVALID_ARGUMENT, std::string(who) + ": too many query tiles");
  a.heads = static_cast<int>(heads);
  a.pairs = static_cast<int>(pairs);
  a.total_items = static_cast<int>(total);
  const ko::DeviceInfo* dinfo = nullptr;
  rc = ko::device_or_fail(&dinfo, who);
  if (rc) return rc;
  const ko::DeviceInfo& info = *dinfo;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Resident CTA pairs (one CTA per SM: shared and tensor memory), found once per device and head dim by the
  // occupancy calculator; the grid is that many pairs or the item count, whichever is smaller.
  static int max_clusters_dev[16][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) dev = 0;
  int* max_clusters = max_clusters_dev[dev];
  auto launch = [&](auto kernel, size_t smem_bytes, int slot) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_bytes));
    if (e != cudaSuccess) return e;
    cfg.dynamicSmemBytes = smem_bytes;
    if (max_clusters[slot] <= 0) {
      cfg.gridDim = dim3(2 * static_cast<unsigned>(info.sm_count / 2));
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
      if (e != cudaSuccess) return e;
      max_clusters[slot] = n > 0 ? n : 1;
    }
    a.n_clusters = static_cast<int>(std::min<int64_t>(total, max_clusters[slot]));
    cfg.gridDim = dim3(2 * static_cast<unsigned>(a.n_clusters));
    return cudaLaunchKernelEx(&cfg, kernel, mq, a);
  };
  cudaError_t e;
  if (head_dim == 64) {
    using C = AttnCfg<64>;
    if (static_cast<int64_t>(C::kSmemBytes) > info.max_smem_optin)
      return ko::fail(KO_ERR_UNSUPPORTED, std::string(who) + ": not enough shared memory on this device");
    e = launch(attention_tf32x3_kernel<64>, C::kSmemBytes, 0);
  } else {
    using C = AttnCfg<32>;
    e = launch(attention_tf32x3_kernel<32>, C::kSmemBytes, 1);
  }
  if (e != cudaSuccess) return ko::fail(static_cast<int>(e), std::string(who) + ": launch failed");
  return ko::check_launch(who);
}
