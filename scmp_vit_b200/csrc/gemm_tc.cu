// SC GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// The SC inner product of row m of a and row n of b is
//     acc[m,n] = sum_d sum_{t < Lp} A'[m,(d,t)] * B'[n,(d,t)]
//     A'[m,(d,t)] = sigma_a(m,d) * [t < k(m,d)]           (enable window)
//     B'[n,(d,t)] = sigma_b(n,d) * [R[d'][t] < c_b(n,d)]   (Sobol/LFSR stream)
// i.e. an exact integer GEMM over an inner dimension of K * Lp with operands in
// {-1, 0, +1}.  Each AND of two stream bits is one int8 multiply-add, each
// popcount is the s32 accumulation in tensor memory.  The operands are never
// stored in HBM: producer warps generate each 128-byte k-block of both
// operands from the int16 codes straight into shared memory, in the
// K-major 128-byte-swizzled layout the UMMA descriptors describe, and one
// thread issues tcgen05.mma for the stage.
//
// CTA tile: 256 rows of a (two 128-row UMMA accumulators) x BN rows of b,
// all 2*BN TMEM columns; 3-stage smem ring; warp 0 issues MMAs, warps 1..16
// generate operands and run the epilogue (rescale + bias + store).  Every wait
// is bounded: on timeout the kernel raises the error flag and drains.
//
// Two producer layouts: row producers (a thread owns one a row and one b row
// of the tile, codes arrive 8 reduction indices per 16-byte load; K % 8 == 0
// and Lp >= 64) and chunk producers (a thread owns one 16-byte chunk column of
// several rows; every other supported shape).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "sc_common.cuh"

namespace scmp {
namespace {

constexpr int kBM = 256;           // a rows per tile (2 x UMMA_M 128)
constexpr int kKB = 128;           // bytes (= inner elements) per k-block
constexpr int kStages = 3;
constexpr int kProducerWarps = 16;
constexpr int kProducers = 32 * kProducerWarps;
constexpr int kThreads = 32 + kProducers;
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // default limit: 2 s per wait

// Limit of every bounded pipeline wait on this device (ns; kTimeoutNs unless
// scmp_debug_set_wait_limit changed it).  Read on the slow path only.
__device__ unsigned long long g_wait_limit_ns = kTimeoutNs;
// Test hook for the give-up path (scmp_debug_hold_producers): while set, the
// operand producers of the e2m1 kernels first wait on g_hold_release, which
// nothing ever sets, so the pipeline waits of their CTA run out.
__device__ int g_hold_producers = 0;
__device__ int g_hold_release = 0;

template <int BN>
struct TcCfg {
  static constexpr uint32_t kStageA = kBM * kKB;  // 32 KB
  static constexpr uint32_t kStageB = BN * kKB;
  static constexpr uint32_t kStage = kStageA + kStageB;
  static constexpr uint32_t kTmemCols = 2 * BN;  // power of two >= 128 (x2 when segmented)
  static constexpr uint32_t kTherm = 2 * 129 * 128;  // enable-window rows (table path)
  // ring depth: 3 x 64 KB for BN = 256, 4 stages for the narrower tiles
  static constexpr int kNS = BN == 256 ? kStages : 4;
  // Dynamic shared memory; kernels without the table leave those 33 KB to L1
  // (at most 196 KB of shared memory keeps a ~60 KB L1 for the pool rows).
  static constexpr size_t smem_bytes(bool table) {
    return (size_t)kNS * kStage + (table ? kTherm : 0) + 1024 /*align*/ + 256;
  }
};

struct TcParams {
  GemmProblem P;
  int lp_log2;      // log2 of the padded stream length Lp (>= 5)
  int shift_pool;   // 1: compare R >> 1 against |c_b| / 2 (bipolar, p == 8)
  int64_t nkb;      // k-blocks per tile = ceil(K * Lp / 128)
  int64_t m_rows;   // rows of a handled per slice (window [0, m_rows))
  int64_t n_rows;   // rows of b handled per slice (window [0, n_rows))
  int64_t tiles_m, tiles_n, tiles;
  unsigned int *error;
  const unsigned char *therm;  // enable-window rows (table path), see therm_table
  int nseg;                    // K segments (1 = unsegmented)
  int kseg;                    // reduction indices per segment
  int64_t nkb_seg;             // k-blocks per segment (nkb = nseg * nkb_seg)
  // Passed at run time so that byte-broadcast products and stage offsets
  // compile to IMADs (the FMA pipe) rather than shifts and adds (the ALU pipe).
  uint32_t rep;          // 0x01010101
  uint32_t stage_bytes;  // TcCfg<BN>::kStage
  int ncols;             // e2m1 CTA pairs: b rows (accumulator columns) per tile
  // e2m1 kernels: MMA k-steps (64 positions each) per 256-position stage that
  // can meet a nonzero window; fewer than 4 when one stream length L < 2^p
  // holds for every row at Lp = 256 (windows end before position
  // ((2^p - 1) L) >> p, e.g. 3 steps at L = 192), so the rest are skipped
  int mma_ksteps = 4;
  // K splits (e2m1 pairs, one segment): prm.tiles = ksplit x tiles_split;
  // split s covers macro steps (8 reduction indices each) [s msplit,
  // min((s + 1) msplit, ldk / 8)) and its tiles write exact int32 counts to
  // part + s part_stride ([batch, M, N]); a reduce kernel rescales their sum.
  int ksplit;
  int msplit;
  int64_t tiles_split;
  int32_t *part;
  int64_t part_stride;
};

// Position of a tile in the launch: its K split, slice and (m, n) block.
struct TileCoord {
  int64_t split, slice, rem;
  int mc0, mc1;  // macro steps of the split
};
template <bool kSplit>
__device__ __forceinline__ TileCoord tile_coord(const TcParams &prm, int64_t tile) {
  TileCoord t;
  const int nmacro = (int)(prm.P.ldk >> 3);
  const int64_t t2 = kSplit ? tile % prm.tiles_split : tile;
  t.split = kSplit ? tile / prm.tiles_split : 0;
  t.slice = t2 / (prm.tiles_m * prm.tiles_n);
  t.rem = t2 % (prm.tiles_m * prm.tiles_n);
  t.mc0 = kSplit ? (int)t.split * prm.msplit : 0;
  t.mc1 = kSplit ? min(t.mc0 + prm.msplit, nmacro) : nmacro;
  return t;
}

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when it gave up (timeout or another thread aborted).
// The limit is re-read on every slow iteration rather than held in registers
// across the loop (waits sit where the producers hold the most live state).
__device__ __forceinline__ unsigned long long wait_limit() {
  return *reinterpret_cast<volatile unsigned long long *>(&g_wait_limit_ns);
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > wait_limit()) {
      *abort = 1;
      return false;
    }
  }
}
// Wait for this thread's own tensor-core work to complete before its TMEM is
// freed: ignores the abort word (MMAs already issued always complete) and
// gives up only after kTimeoutNs.
__device__ __forceinline__ void mbar_wait_own(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long t0 = now_ns();
  while (!mbar_try_wait(bar, parity) && now_ns() - t0 <= kTimeoutNs) {
  }
}
// Test hook: with g_hold_producers set, wait on a flag that nothing sets until
// the wait limit runs out (or the CTA aborts); false = give up.
__device__ __forceinline__ bool producers_released(volatile int *abort) {
  if (!*reinterpret_cast<volatile int *>(&g_hold_producers)) return true;
  const unsigned long long t0 = now_ns();
  while (!*reinterpret_cast<volatile int *>(&g_hold_release)) {
    if (*abort) return false;
    if (now_ns() - t0 > wait_limit()) {
      *abort = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// ---- CTA pairs (cta_group::2): the even CTA of a 2-CTA cluster issues the
// MMAs for both; every other wait on a peer is an mbarrier with a bound.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `addr` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Cluster-scope release: issued only by threads with no global loads in
// flight (a release waits for them), never by the producers per k-block.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cl(uint64_t *bar, uint32_t parity, volatile int *abort) {
  if (mbar_try_wait_cl(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (true) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > wait_limit()) {
      *abort = 1;
      return false;
    }
  }
}
// mbar_wait_own with cluster-scope acquire (pair MMAs arrive from the pair).
__device__ __forceinline__ void mbar_wait_own_cl(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait_cl(bar, parity)) return;
  const unsigned long long t0 = now_ns();
  while (!mbar_try_wait_cl(bar, parity) && now_ns() - t0 <= kTimeoutNs) {
  }
}
// Both CTAs of the pair reach this point (every path to it is bounded).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tc_mma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Completion of this thread's pair MMAs arrives on `bar` in both CTAs (the
// barrier sits at the same shared-memory offset in each).
__device__ __forceinline__ void tc_commit_pair_both(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair_local(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// ---- TMA (prepacked b): a plain 2-D tiled load into this CTA's shared
// memory, completing bytes on an mbarrier (no multicast).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// L2 prefetch of one tensor-map tile of this GPU's memory (no shared memory,
// no multicast): the prepacked-b loader asks for a k-block some stages
// before its load, so that the load finds it in L2.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// 32 consecutive TMEM columns of this warp's 32 lanes (lane i -> row i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                 "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                   taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
               "r"(v[7])
               : "memory");
}

// K-major, 128-byte-swizzled UMMA shared-memory descriptor: 8-row atoms of
// 128 B (1024 B apart), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);        // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused here)
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B
  return d;
}

// The descriptor of addr + bytes from that of addr: the start-address field
// holds (addr & 0x3FFFF) >> 4 in 14 bits, so adding bytes >> 4 is exact while
// addr + bytes stays below 256 KB and bytes is a multiple of 16 (every tile
// offset here).  One 64-bit add instead of rebuilding the descriptor: the
// MMA thread shares its SM sub-partition with busy producer warps, and its
// instructions per stage are on the tensor pipe's critical path.
__device__ __forceinline__ uint64_t desc_add(uint64_t desc, uint32_t bytes) {
  return desc + (uint64_t)(bytes >> 4);
}

// Instruction descriptor: s8 x s8 -> s32, K-major A and B, M = 128, N = BN.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_i8() {
  return (2u << 4)                      // D format S32
         | (1u << 7)                    // A format S8
         | (1u << 10)                   // B format S8
         | ((uint32_t)(BN >> 3) << 17)  // N >> 3
         | ((uint32_t)(128 >> 4) << 24);  // M >> 4
}

// Byte offset of 16-byte chunk `c` of row `r` in a SW128 K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// ------------------------------------------------------------------ kernel

// Producer kinds.
constexpr int kProdChunks = 0;  // thread = (row group, 16-byte chunk); windows by byte compares
constexpr int kProdTable = 1;   // as kProdChunks, enable windows copied from a smem table
constexpr int kProdRows = 2;    // thread = one a row and one b row (see produce_rows)

// Shared-memory barriers and the abort word (carved after the stage ring).
struct Bars {
  uint64_t *full, *empty, *tfull, *tempty, *drain, *epi;
  volatile int *abort;
  // CTA pairs: the even CTA's peer-stage barriers pfull[] (arrived on by the
  // odd CTA's forwarder thread) and tempty, as shared::cluster addresses
  uint64_t *pfull;
  uint32_t pfull_cl, tempty_cl;
};

// Producer-side pipeline position (per thread).
struct ProdState {
  int stage;
  uint32_t phase;
  int64_t g;  // drain counter: one per (tile, segment), as on the MMA side
};

// Every lane polls (one issue slot per poll, like a single lane, but the warp
// never diverges); the lanes agree on the outcome.
__device__ __forceinline__ bool acquire_stage(const Bars &b, const ProdState &st, int lane) {
  (void)lane;
  const bool ok = mbar_wait(&b.empty[st.stage], st.phase ^ 1, b.abort);
  return __all_sync(0xffffffffu, ok);
}
// Stage s known at compile time (row producers whose macro step is a whole
// number of ring turns).
__device__ __forceinline__ bool acquire_at(const Bars &b, int s, uint32_t phase) {
  const bool ok = mbar_wait(&b.empty[s], phase ^ 1, b.abort);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ void publish_at(const Bars &b, int s, int lane) {
  fence_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(&b.full[s]);
}
__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Every lane publishes its writes to the async proxy, then one lane per warp
// arrives (the release covers the warp's writes through __syncwarp).
template <int NS = kStages>
__device__ __forceinline__ void publish_stage(const Bars &b, ProdState &st, int lane) {
  fence_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(&b.full[st.stage]);
  if (++st.stage == NS) {
    st.stage = 0;
    st.phase ^= 1;
  }
}

// Segmented tiles: 16 accumulator columns of this warp's 32 rows after
// segment `sd` -- rescale the counts (int32, or with kF32 the e2m1 tiles'
// exact fp32 counts) with the segment's scales and add the fp32 sum of the
// earlier segments.  acc_col / run_col: TMEM columns of the counts and of the
// running sums; gn0: the b row of the first column.  Result in y (fp32 bits).
template <bool kF32, int W = 16>
__device__ __forceinline__ void seg_chunk16(const TcParams &prm, uint32_t lanebase, int lane,
                                            int sd, uint32_t acc_col, uint32_t run_col,
                                            int64_t gn0, int64_t grow, bool row_ok, int L,
                                            int64_t slice_b, uint32_t (&y)[W]) {
  static_assert(W == 8 || W == 16, "8 or 16 columns");
  const GemmProblem &P = prm.P;
  float sa = 0.f;
  int za = 0, rsa = 0;
  if (row_ok && L > 0) {
    const int64_t ra = grow * prm.nseg + sd;
    sa = P.qa.scale[ra];
    za = P.qa.zero[ra];
    rsa = P.qa.rowsum[ra];
  }
  const int64_t gn = gn0 + (lane & (W - 1));
  float sbl = 0.f;
  int zbl = 0, rsbl = 0;
  if (gn < prm.n_rows) {
    const int64_t rb = (slice_b * P.N + gn) * prm.nseg + sd;
    sbl = P.qb.scale[rb];
    zbl = P.qb.zero[rb];
    rsbl = P.qb.rowsum[rb];
  }
  uint32_t f[W];
  if constexpr (W == 16) {
    tmem_ld16(lanebase + acc_col, y);
    if (sd > 0) tmem_ld16(lanebase + run_col, f);
  } else {
    tmem_ld8(lanebase + acc_col, y);
    if (sd > 0) tmem_ld8(lanebase + run_col, f);
  }
  // the row's rescale factor F = 2^(2p) / (u L), once per call (bit-identical
  // to computing it per element: it depends on the row only)
  const bool live = row_ok && L > 0;
  const float F = live ? sc_rescale_factor(P.mode, P.prec, L) : 0.0f;
  const bool unipolar = P.mode != SCMP_BIPOLAR;  // bipolar needs no zero points
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const float sb = __shfl_sync(0xffffffffu, sbl, i);
    int zb = 0, rsb = 0;
    if (unipolar) {
      zb = __shfl_sync(0xffffffffu, zbl, i);
      rsb = __shfl_sync(0xffffffffu, rsbl, i);
    }
    const int32_t cnt = kF32 ? __float2int_rn(__uint_as_float(y[i])) : (int32_t)y[i];
    const float r = live ? sc_rescale_f(P.mode, F, cnt, prm.kseg, sa, za, rsa, sb, zb, rsb) : 0.0f;
    y[i] = __float_as_uint(sd == 0 ? r : __fadd_rn(__uint_as_float(f[i]), r));
  }
}

// The 2-accumulator layout of the int8 tiles: half `h` of 32-column chunk
// `cc` of accumulator acc_j, running sums in TMEM columns 2 BN ..
template <int BN>
__device__ __forceinline__ void seg_chunk(const TcParams &prm, uint32_t tmem_base, int lane,
                                          int sd, int cc, int h, int acc_j, int quarter,
                                          int64_t grow, bool row_ok, int L, int64_t slice_b,
                                          int64_t n0, uint32_t (&y)[16]) {
  const uint32_t col = (uint32_t)(acc_j * BN + cc * 32 + h * 16);
  seg_chunk16<false>(prm, tmem_base + ((uint32_t)(quarter * 32) << 16), lane, sd, col,
                     (uint32_t)(2 * BN) + col, n0 + cc * 32 + h * 16, grow, row_ok, L, slice_b, y);
}

// End of a non-final segment: wait for its MMAs, fold the int32 counts into
// the fp32 running sums in TMEM, hand the accumulators back to the MMA warp.
template <int BN>
__device__ bool segment_drain(const TcParams &prm, const Bars &b, ProdState &st,
                              uint32_t tmem_base, int warp, int lane, int sd, int64_t slice,
                              int64_t slice_b, int64_t m0, int64_t n0) {
  const GemmProblem &P = prm.P;
  if (!mbar_wait(b.tfull, (uint32_t)(st.g & 1), b.abort)) return false;
  tc_fence_after();
  const int pw = warp - 1;
  const int quarter = warp & 3;
  const int acc_j = (pw >> 2) & 1;
  const int col_half = pw >> 3;
  const int64_t gm = m0 + acc_j * 128 + quarter * 32 + lane;
  const bool row_ok = gm < prm.m_rows;
  const int64_t grow = slice * P.M + gm;
  const int L = row_ok ? row_stream_len(P, slice, grow) : -1;
  const uint32_t lanebase = tmem_base + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
  for (int cc = col_half * (BN / 64); cc < (col_half + 1) * (BN / 64); ++cc) {
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      uint32_t y[16];
      seg_chunk<BN>(prm, tmem_base, lane, sd, cc, h, acc_j, quarter, grow, row_ok, L, slice_b, n0,
                    y);
      tmem_st16(lanebase + (uint32_t)(2 * BN + acc_j * BN + cc * 32 + h * 16), y);
    }
  }
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  tc_fence_before();
  mbar_arrive(b.tempty);
  ++st.g;
  return true;
}

// End of a non-final segment of a one-accumulator e2m1 pair tile (the CTA's
// 128 a rows in TMEM lanes, ncols fp32 count columns): wait for the segment's
// MMAs, fold the counts into the fp32 running sums in TMEM columns
// [ncols, 2 ncols), then hand the accumulator back to the pair's MMA thread
// (one cluster arrival per CTA once all of its producers are done).  n0: the
// tile's first b row (the accumulator covers both CTAs' b rows).
__device__ bool segment_drain_pair(const TcParams &prm, const Bars &b, ProdState &st,
                                   uint32_t tmem_base, int warp, int lane, int sd, int64_t slice,
                                   int64_t slice_b, int64_t m0, int64_t n0) {
  const GemmProblem &P = prm.P;
  const int ncols = prm.ncols;
  if (!mbar_wait(b.tfull, (uint32_t)(st.g & 1), b.abort)) return false;
  tc_fence_after();
  const int pw = warp - 1;
  const int quarter = warp & 3;  // the TMEM lanes this warp may access
  const int64_t gm = m0 + quarter * 32 + lane;
  const bool row_ok = gm < prm.m_rows;
  const int64_t grow = slice * P.M + gm;
  const int L = row_ok ? row_stream_len(P, slice, grow) : -1;
  const uint32_t lanebase = tmem_base + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
  for (int c = 8 * (pw >> 2); c < ncols; c += 32) {  // the quarter's 4 warps share the columns
    uint32_t y[8];
    seg_chunk16<true, 8>(prm, lanebase, lane, sd, (uint32_t)c, (uint32_t)(ncols + c), n0 + c,
                         grow, row_ok, L, slice_b, y);
    tmem_st8(lanebase + (uint32_t)(ncols + c), y);
  }
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  tc_fence_before();
  mbar_arrive(b.epi);
  if (!mbar_wait(b.epi, (uint32_t)(st.g & 1), b.abort)) return false;
  if (threadIdx.x == 32) mbar_arrive_cluster(b.tempty_cl);
  ++st.g;
  return true;
}

// ---------------------------------------------------------------------------
// Chunk producers: thread pt fills 16-byte chunk `chunk` of a-rows rsub + 64 i
// (i < 4) and b-rows rsub + 64 i (i < BN / 64) of every k-block.  Codes and
// pool bytes of k-block kb + 1 are loaded while k-block kb is generated.
// Handles every supported shape (ragged K, Lp = 32).
template <int BN, bool kBulkA, bool kSeg>
__device__ bool produce_chunks(const TcParams &prm, const Bars &b, ProdState &st,
                               uint32_t smem_s, uint32_t therm_u, uint32_t tmem_base, int warp,
                               int lane, int64_t slice, int64_t slice_b, int64_t m0, int64_t n0) {
  using Cfg = TcCfg<BN>;
  const GemmProblem &P = prm.P;
  constexpr int kRowsA = kBM / 64;             // 4
  constexpr int kNB = BN >= 64 ? BN / 64 : 1;  // b rows per thread
  const int pt = threadIdx.x - 32;             // 0 .. kProducers-1
  const int chunk = pt & 7;
  const int rsub = pt >> 3;  // 0 .. 63
  const int T = 1 << P.prec;
  // 32-bit index math in the k-block loop: K * Lp < 2^31 and pool_dims >= K
  // are guaranteed by the launcher (tc_supported / launch_gemm_tc).
  const int lg = prm.lp_log2;
  const int Lp32 = 1 << lg;
  const int K32 = (int)P.K;
  // pool row of reduction index d: d itself, or d's index inside its segment
  // (segmented problems use a (k_segment, p) pool shared by every segment)
  auto pool_row = [&](int d) -> int { return kSeg ? d % prm.kseg : d; };
  const uint32_t tw0 = 0x03020100u, tw1 = 0x07060504u, tw2 = 0x0B0A0908u, tw3 = 0x0F0E0D0Cu;
  // byte offsets of this thread's chunks inside the A / B stage (row r = rsub + 64 i)
  const uint32_t offA0 = sw128_offset(rsub, chunk);

  int Lrow[kRowsA];
  const int16_t *arow[kRowsA];
#pragma unroll
  for (int i = 0; i < kRowsA; ++i) {
    const int64_t gm = m0 + rsub + 64 * i;
    Lrow[i] = 0;
    arow[i] = P.qa.code;  // dummy, never read when Lrow = 0 / invalid
    if (gm < prm.m_rows) {
      const int64_t grow = slice * P.M + gm;
      Lrow[i] = row_stream_len(P, slice, grow);
      arow[i] = P.qa.code + grow * P.ldk;
    }
  }
  bool bval[kNB];
  const int16_t *brow[kNB];
#pragma unroll
  for (int i = 0; i < kNB; ++i) {
    const int64_t gn = n0 + rsub + 64 * i;
    bval[i] = (rsub + 64 * i < BN) && gn < prm.n_rows;
    brow[i] = bval[i] ? P.qb.code + (slice_b * P.N + gn) * P.ldk : P.qb.code;
  }
  // ---- prefetch k-block 0
  int16_t ca_n[kRowsA], cb_n[kNB];
  uint4 rr_n = make_uint4(0, 0, 0, 0);
  int t0_n = 0;
  {
    const int i0 = chunk * 16;
    const int d = i0 >> lg;
    t0_n = i0 & (Lp32 - 1);
    const bool dv = d < K32;
#pragma unroll
    for (int i = 0; i < kRowsA; ++i)
      ca_n[i] = (dv && Lrow[i] != 0) ? __ldg(arow[i] + d) : (int16_t)0;
#pragma unroll
    for (int i = 0; i < kNB; ++i) cb_n[i] = (dv && bval[i]) ? __ldg(brow[i] + d) : (int16_t)0;
    if (dv) rr_n = __ldg(reinterpret_cast<const uint4 *>(P.pool + (pool_row(d) * T + t0_n)));
  }
  for (int64_t kb = 0; kb < prm.nkb; ++kb) {
    int16_t ca[kRowsA], cb[kNB];
#pragma unroll
    for (int i = 0; i < kRowsA; ++i) ca[i] = ca_n[i];
#pragma unroll
    for (int i = 0; i < kNB; ++i) cb[i] = cb_n[i];
    uint4 rr = rr_n;
    const int t0 = t0_n;
    // k-block start inside its reduction index (table path: one d per k-block)
    const int t0_blk = ((int)kb * kKB) & (Lp32 - 1);
    if (kb + 1 < prm.nkb) {
      const int i0 = ((int)kb + 1) * kKB + chunk * 16;
      const int d = i0 >> lg;
      t0_n = i0 & (Lp32 - 1);
      const bool dv = d < K32;
#pragma unroll
      for (int i = 0; i < kRowsA; ++i)
        ca_n[i] = (dv && Lrow[i] != 0) ? __ldg(arow[i] + d) : (int16_t)0;
#pragma unroll
      for (int i = 0; i < kNB; ++i) cb_n[i] = (dv && bval[i]) ? __ldg(brow[i] + d) : (int16_t)0;
      rr_n = dv ? __ldg(reinterpret_cast<const uint4 *>(P.pool + (pool_row(d) * T + t0_n)))
                : make_uint4(0, 0, 0, 0);
    }
    if (prm.shift_pool) {
      rr.x = (rr.x >> 1) & 0x7F7F7F7Fu; rr.y = (rr.y >> 1) & 0x7F7F7F7Fu;
      rr.z = (rr.z >> 1) & 0x7F7F7F7Fu; rr.w = (rr.w >> 1) & 0x7F7F7F7Fu;
    }
    // byte j of (u * 0x01010101 + base_w) is 0x7F + u - R[t0+4w+j]; its top
    // bit is [R < u] (no borrows: u, R < 128), read by the sign-replicating
    // byte permute
    const uint32_t rb0 = 0x7F7F7F7Fu - rr.x, rb1 = 0x7F7F7F7Fu - rr.y;
    const uint32_t rb2 = 0x7F7F7F7Fu - rr.z, rb3 = 0x7F7F7F7Fu - rr.w;
    if (!acquire_stage(b, st, lane)) return false;
    const uint32_t sa_s = smem_s + (uint32_t)st.stage * Cfg::kStage + offA0;
    const uint32_t sb_s = sa_s + Cfg::kStageA;
    // ---- A: enable windows, sigma * [t < k]
    if constexpr (kBulkA) {
      // one k-block = 128 stream positions of one reduction index: copy
      // chunk `chunk` of the window row (sign, q) from the smem table
#pragma unroll
      for (int i = 0; i < kRowsA; ++i) {
        const int c = ca[i];
        const int k = (abs(c) * Lrow[i]) >> P.prec;
        const int q = min(max(k - t0_blk, 0), 128);
        const uint4 w =
            ld_shared_v4(therm_u + (uint32_t)((((c < 0 ? 129 : 0) + q) << 7) + (chunk << 4)));
        st_shared_v4(sa_s + i * 8192, w.x, w.y, w.z, w.w);
      }
    }
#pragma unroll
    for (int i = 0; i < (kBulkA ? 0 : kRowsA); ++i) {
      const int c = ca[i];
      const int k = (abs(c) * Lrow[i]) >> P.prec;
      const uint32_t q = (uint32_t)min(max(k - t0, 0), 16);
      const uint32_t sm = (uint32_t)(c >> 31) | 0x01010101u;
      // byte j of (q * 0x01010101 + 0x7F7F7F7F - tw) is 0x7F + q - j: top bit = [j < q]
      st_shared_v4(sa_s + i * 8192,  // +64 rows = 8 atoms
                   prmt(q * 0x01010101u + (0x7F7F7F7Fu - tw0), 0u, 0xBA98u) & sm,
                   prmt(q * 0x01010101u + (0x7F7F7F7Fu - tw1), 0u, 0xBA98u) & sm,
                   prmt(q * 0x01010101u + (0x7F7F7F7Fu - tw2), 0u, 0xBA98u) & sm,
                   prmt(q * 0x01010101u + (0x7F7F7F7Fu - tw3), 0u, 0xBA98u) & sm);
    }
    // ---- B: streams, sigma * [R[d'][t] < c_b]
#pragma unroll
    for (int i = 0; i < kNB; ++i) {
      if (rsub + 64 * i >= BN) break;
      const int c = cb[i];
      const uint32_t u = (uint32_t)(abs(c) >> prm.shift_pool);
      const uint32_t sm = (uint32_t)(c >> 31) | 0x01010101u;
      st_shared_v4(sb_s + i * 8192,
                   prmt(u * 0x01010101u + rb0, 0u, 0xBA98u) & sm,
                   prmt(u * 0x01010101u + rb1, 0u, 0xBA98u) & sm,
                   prmt(u * 0x01010101u + rb2, 0u, 0xBA98u) & sm,
                   prmt(u * 0x01010101u + rb3, 0u, 0xBA98u) & sm);
    }
    publish_stage<Cfg::kNS>(b, st, lane);
    if constexpr (kSeg) {
      if ((kb + 1) % prm.nkb_seg == 0 && kb + 1 < prm.nkb) {
        // ---- end of a non-final segment
        if (!segment_drain<BN>(prm, b, st, tmem_base, warp, lane, (int)(kb / prm.nkb_seg), slice,
                               slice_b, m0, n0))
          return false;
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Row producers (K % 8 == 0, Lp >= 64).  Thread pt owns a-row pt % 256 (its
// chunks 4 (pt / 256) .. + 3) and b-row pt % BN (its BN / 64 chunks starting
// at (BN / 64) (pt / BN)), so a warp covers 32 consecutive rows of one
// operand and each code is turned into a window length / threshold once per
// k-block, not once per chunk.  Codes arrive 8 reduction indices at a time
// (one 16-byte load per row per macro step of G = Lp / 16 k-blocks).
//
// Bytes are produced four at a time with one IMAD, one byte permute and one
// AND: for a chunk starting at stream position t0,
//   a: word j = sign(0x7F + (k - t0) - (4 j + b)) for bytes b < 4, i.e. the
//      top bit of byte b is [t0 + 4 j + b < k] (k - t0 in [-112, 128], so no
//      byte under- or overflows);
//   b: word j = sign(u + PC[d'][t0 + 4 j + b]) with PC = 0x7F - (R >> shift),
//      top bit [R >> shift < u] (u < 128).
// sign(x) replicates each byte's top bit (prmt 0xBA98) and is ANDed with
// 0x01010101 (sigma = +1) or 0xFFFFFFFF (sigma = -1).
__device__ __forceinline__ uint32_t mad_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// 16 bytes of codes read once per macro step: no L1 allocation, so the pool
// complement rows the producers re-read stay resident
__device__ __forceinline__ uint4 ld_stream_v4(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
// code of reduction index `idx` (0..7) of a macro step: int16 lane of the
// 16-byte code load
__device__ __forceinline__ int code_of(const uint4 &v, int idx) {
  const uint32_t w = word_of(v, idx >> 1);
  return (idx & 1) ? ((int)w >> 16) : (int)(int16_t)(w & 0xFFFFu);
}
// code of index 2 j + e (e in {0, 1} known only at run time): sh = 16 - 16 e
__device__ __forceinline__ int code_of_rt(const uint4 &v, int j, uint32_t sh) {
  return (int)(word_of(v, j) << sh) >> 16;
}

// BN = b rows this CTA generates (starting at n0); CTA pairs (kPair) run NS
// stages.
// kNoB: b arrives by TMA from a prepacked buffer; only the a rows are generated.
// kSparseA: a warp stores zeros without arithmetic for a chunk that lies past
// every window of its 32 rows (short windows dominate in Attn@V, whose a rows
// are softmax probabilities); exact, since such bytes are zero anyway.
template <int BN, int LG, bool kSeg, int NS, bool kPair = false, bool kNoB = false,
          bool kSparseA = false>
__device__ bool produce_rows(const TcParams &prm, const Bars &b, ProdState &st, uint32_t smem_s,
                             uint32_t tmem_base, int warp, int lane, int64_t slice,
                             int64_t slice_b, int64_t m0, int64_t n0) {
  static_assert(LG >= 6 && LG <= 8, "row producers need 64 <= Lp <= 256");
  static_assert(!(kSeg && kPair), "CTA pairs run unsegmented problems");
  using Cfg = TcCfg<BN>;
  const GemmProblem &P = prm.P;
  constexpr int NBC = BN / 64;          // b chunks per thread
  constexpr int G = (1 << LG) / 16;     // k-blocks per macro step (8 reduction indices)
  constexpr int LPB = 1 << LG;          // pool complement row stride (bytes)
  // a macro step that is a whole number of ring turns starts at stage 0:
  // stage and phase of each k-block are then known at compile time
  constexpr bool kStatic = (G % NS) == 0;
  constexpr uint32_t kStageBytes = Cfg::kStage;
  const int pt = threadIdx.x - 32;
  const int ra = pt & 255;              // a row of the tile
  const int hA = pt >> 8;               // a chunks 4 hA .. 4 hA + 3
  const int rbn = pt & (BN - 1);        // b row of the tile
  const int cB0 = NBC * (pt / BN);      // first b chunk
  // rows (an invalid row reads the last valid row: its outputs are never
  // stored; with CTA pairs a whole half tile can lie past the last row)
  const int64_t gmA = m0 + ra;
  const bool vA = gmA < prm.m_rows;
  const int64_t growA = slice * P.M + (vA ? gmA : prm.m_rows - 1);
  int Lg = 0;
  if (vA) {
    const int L = row_stream_len(P, slice, growA);
    Lg = L > 0 ? L : 0;
  }
  const int64_t gnB = n0 + rbn;
  const int64_t growB = slice_b * P.N + (gnB < prm.n_rows ? gnB : prm.n_rows - 1);
  const uint4 *pa = reinterpret_cast<const uint4 *>(P.qa.code + growA * P.ldk);
  const uint4 *pb = reinterpret_cast<const uint4 *>(P.qb.code + growB * P.ldk);
  // shared-memory addresses of this thread's chunks in stage 0
  uint32_t sA[4], sB[NBC];
#pragma unroll
  for (int i = 0; i < 4; ++i) sA[i] = smem_s + sw128_offset(ra, 4 * hA + i);
#pragma unroll
  for (int i = 0; i < NBC; ++i) sB[i] = smem_s + Cfg::kStageA + sw128_offset(rbn, cB0 + i);
  // stream position of the first a chunk inside its reduction index (or
  // half index for Lp = 256), and of the first b chunk
  const int t0A = LG >= 7 ? 64 * hA : 0;
  const int t0B = LG >= 7 ? 16 * cB0 : 16 * (cB0 & 3);
  // Lp = 64: a chunks lie in index 2 j + hA, b chunks in 2 j + (cB0 >> 2)
  const uint32_t shA = 16u - 16u * (uint32_t)hA;
  const uint32_t shB = 16u - 16u * (uint32_t)(cB0 >> 2);
  const uint32_t rep = prm.rep;           // 0x01010101
  const uint32_t stage_bytes = prm.stage_bytes;
  const int prec = P.prec;
  const int shift = prm.shift_pool;
  const int nmacro = (int)(P.ldk >> 3);  // zero-padded indices past K add nothing
  const int msteps_seg = kSeg ? prm.kseg >> 3 : 0;  // macro steps per segment
  // Pool complement rows are LPB bytes apart (the table is laid out with the
  // padded stream length as row stride), so k-block j of a macro step reads
  // its b chunks at pcm + 128 j for every Lp: Lp = 128 one row per k-block,
  // Lp = 256 half a row, Lp = 64 the row 2 j + (cB0 >> 2).
  const uint8_t *pc_thr = P.pool_comp + t0B + (LG == 6 ? 64 * (cB0 >> 2) : 0);
  // pool rows one segment (or the whole K) spans
  const int prow_lim = kSeg ? prm.kseg : (int)P.ldk;
  // the 8 rows (G lines of 128 B) of a macro step are pulled into L1 one
  // macro step ahead, one line per lane
  auto prefetch_macro = [&](int prow) {
    if (lane < G && prow < prow_lim) prefetch_l1(P.pool_comp + (size_t)prow * LPB + 128 * lane);
  };
  int pbase = 0;  // pool row of the macro step's first reduction index
  int mseg = 0;   // macro steps done in the current segment
  uint4 ca_n = ld_stream_v4(pa), cb_n = make_uint4(0, 0, 0, 0);
  if constexpr (!kNoB) {
    cb_n = ld_stream_v4(pb);
    prefetch_macro(0);
  }
#pragma unroll 1
  for (int mc = 0; mc < nmacro; ++mc) {
    const uint4 ca = ca_n, cb = cb_n;
    if (mc + 1 < nmacro) {
      ca_n = ld_stream_v4(pa + mc + 1);
      if constexpr (!kNoB) cb_n = ld_stream_v4(pb + mc + 1);
    }
    if constexpr (!kNoB) prefetch_macro((kSeg && mseg + 1 == msteps_seg) ? 0 : pbase + 8);
    const uint8_t *pcm = pc_thr + (size_t)pbase * LPB;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      // ---- b: pool complement bytes of this k-block's b chunks
      const uint8_t *pc = pcm + 128 * j;
      uint4 pcw[NBC];
#pragma unroll
      for (int i = 0; i < NBC; ++i)
        pcw[i] = kNoB ? make_uint4(0, 0, 0, 0) : __ldg(reinterpret_cast<const uint4 *>(pc) + i);
      // ---- a: window length of this k-block's reduction index
      const int codeA = LG == 6 ? code_of_rt(ca, j, shA) : code_of(ca, LG == 8 ? (j >> 1) : j);
      int k = (abs(codeA) * Lg) >> prec;
      if (LG == 8) k = (j & 1) ? max(k - 128, 0) : min(k, 128);
      const uint32_t kbase = (uint32_t)(k - t0A);
      const uint32_t smA = (uint32_t)(codeA >> 31) | 0x01010101u;
      const int codeB = LG == 6 ? code_of_rt(cb, j, shB) : code_of(cb, LG == 8 ? (j >> 1) : j);
      const uint32_t u = (uint32_t)(abs(codeB) >> shift);
      const uint32_t smB = (uint32_t)(codeB >> 31) | 0x01010101u;
      uint32_t soff;  // byte offset of this k-block's stage
      if constexpr (kStatic) {
        if (!acquire_at(b, j % NS, st.phase ^ (uint32_t)((j / NS) & 1))) return false;
        soff = (uint32_t)(j % NS) * kStageBytes;
      } else {
        if (!acquire_stage(b, st, lane)) return false;
        soff = mad_u32((uint32_t)st.stage, stage_bytes, 0u);
      }
      // largest k - t0A over the warp's rows (the warp shares hA, so t0A)
      const int kbmax = kSparseA ? __reduce_max_sync(0xffffffffu, (int)kbase) : 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // chunk 4 hA + i starts at t0A + 16 i: k - t0 = kbase - 16 i
        const uint32_t kc = kbase - 16u * (uint32_t)i;
        if (kSparseA && kbmax <= 16 * i) {  // warp-uniform: no window reaches this chunk
          st_shared_v4(sA[i] + soff, 0u, 0u, 0u, 0u);
          continue;
        }
        st_shared_v4(sA[i] + soff,
                     prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x03020100u), 0u, 0xBA98u) & smA,
                     prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x07060504u), 0u, 0xBA98u) & smA,
                     prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x0B0A0908u), 0u, 0xBA98u) & smA,
                     prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x0F0E0D0Cu), 0u, 0xBA98u) & smA);
      }
#pragma unroll
      for (int i = 0; i < (kNoB ? 0 : NBC); ++i) {
        st_shared_v4(sB[i] + soff,
                     prmt(mad_u32(u, rep, pcw[i].x), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].y), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].z), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].w), 0u, 0xBA98u) & smB);
      }
      if constexpr (kStatic)
        publish_at(b, j % NS, lane);
      else
        publish_stage<NS>(b, st, lane);
    }
    if constexpr (kStatic) {
      if ((G / NS) & 1) st.phase ^= 1u;  // st.stage stays 0
    }
    pbase += 8;
    if constexpr (kSeg) {
      if (++mseg == msteps_seg) {
        mseg = 0;
        pbase = 0;
        // ---- end of a segment (the last one drains in the epilogue)
        if (mc + 1 < nmacro &&
            !segment_drain<BN>(prm, b, st, tmem_base, warp, lane, (mc + 1) / msteps_seg - 1,
                               slice, slice_b, m0, n0))
          return false;
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Narrow tiles with the window operand in tensor memory (tcgen05.mma reading
// A from TMEM).  With BN <= 128 the 256 a rows are most of the operand bytes;
// in shared memory they cost a 32 KB store plus a 32 KB MMA read per k-block,
// the bandwidth that bounds those tiles.  Here each producer thread writes its
// 64 bytes of an a row straight into its TMEM lane (one tcgen05.st of 16
// columns); only the BN b rows go through shared memory.
//
// TMEM columns: [0, 2 BN) the two int32 accumulators (a rows 0-127 / 128-255),
// then kTsStages stages of 64 columns: half h (a rows 128 h .. + 127, one per
// lane) at +32 h, its 128 bytes of k-block as 32 columns of 4 int8 each.
constexpr int kTsStages = 4;
constexpr uint32_t kEpiStagingBytes =  // tile_epilogue's transpose, row records, row factors
    kProducerWarps * 32 * 33 * 4 + kProducerWarps * 32 * 16 + kProducerWarps * 32 * 4;

template <int BN>
struct TsCfg {
  static constexpr uint32_t kStageB = BN * kKB;
  // the ring doubles as the epilogue's staging area
  static constexpr uint32_t kRing =
      ((kTsStages * kStageB > kEpiStagingBytes ? kTsStages * kStageB : kEpiStagingBytes) + 1023) &
      ~1023u;
  static constexpr uint32_t kAcol = 2 * BN;   // first window-operand column
  static constexpr uint32_t kAStageCols = 64;  // 256 rows x 128 bytes over 128 lanes
  static_assert(kAcol + kTsStages * kAStageCols <= 512, "accumulators + window stages fit TMEM");
  static constexpr size_t smem_bytes = (size_t)kRing + 1024 /*align*/ + 256;
};

__device__ __forceinline__ void tc_mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Row producers for the TMEM window operand.  TMEM lane quarters follow the
// warp (warp w reaches lanes 32 (w % 4) ..), so producer warp pw = w - 1
// generates a rows 128 h + 32 (w % 4) + lane, h = (pw / 4) % 2, and the half
// 64 e .. 64 e + 63 of their k-block bytes, e = pw / 8.  The b rows and the
// code / pool-complement streaming are those of produce_rows.  A chunk that
// lies past every window of the warp's 32 rows is zero and one that lies
// inside all of them is sigma in every byte; neither needs arithmetic.
template <int BN, int LG>
__device__ bool produce_rows_ts(const TcParams &prm, const Bars &b, ProdState &st, uint32_t smem_s,
                                uint32_t tmem_base, int warp, int lane, int64_t slice,
                                int64_t slice_b, int64_t m0, int64_t n0) {
  static_assert(LG >= 6 && LG <= 8, "row producers need 64 <= Lp <= 256");
  using Cfg = TsCfg<BN>;
  constexpr int NS = kTsStages;
  const GemmProblem &P = prm.P;
  constexpr int NBC = BN / 64;       // b chunks per thread
  constexpr int G = (1 << LG) / 16;  // k-blocks per macro step (8 reduction indices)
  constexpr int LPB = 1 << LG;       // pool complement row stride (bytes)
  static_assert(G % NS == 0, "a macro step is a whole number of ring turns");
  const int pt = threadIdx.x - 32;
  const int pw = warp - 1;
  const int quarter = warp & 3;
  const int hA = pw >> 3;                                  // a bytes 64 hA .. + 63
  const int ra = ((pw >> 2) & 1) * 128 + quarter * 32 + lane;  // a row of the tile
  const int rbn = pt & (BN - 1);
  const int cB0 = NBC * (pt / BN);
  const int64_t gmA = m0 + ra;
  const bool vA = gmA < prm.m_rows;
  const int64_t growA = slice * P.M + (vA ? gmA : prm.m_rows - 1);
  int Lg = 0;
  if (vA) {
    const int L = row_stream_len(P, slice, growA);
    Lg = L > 0 ? L : 0;
  }
  const int64_t gnB = n0 + rbn;
  const int64_t growB = slice_b * P.N + (gnB < prm.n_rows ? gnB : prm.n_rows - 1);
  const uint4 *pa = reinterpret_cast<const uint4 *>(P.qa.code + growA * P.ldk);
  const uint4 *pb = reinterpret_cast<const uint4 *>(P.qb.code + growB * P.ldk);
  // this warp's 16 columns of stage 0 (lane field = the quarter's first lane)
  const uint32_t tA = tmem_base + ((uint32_t)(quarter * 32) << 16) + Cfg::kAcol +
                      (uint32_t)(((pw >> 2) & 1) * 32 + hA * 16);
  uint32_t sB[NBC];
#pragma unroll
  for (int i = 0; i < NBC; ++i) sB[i] = smem_s + sw128_offset(rbn, cB0 + i);
  const int t0A = LG >= 7 ? 64 * hA : 0;
  const int t0B = LG >= 7 ? 16 * cB0 : 16 * (cB0 & 3);
  const uint32_t shA = 16u - 16u * (uint32_t)hA;
  const uint32_t shB = 16u - 16u * (uint32_t)(cB0 >> 2);
  const uint32_t rep = prm.rep;  // 0x01010101
  const int prec = P.prec;
  const int shift = prm.shift_pool;
  const int nmacro = (int)(P.ldk >> 3);
  const uint8_t *pc_thr = P.pool_comp + t0B + (LG == 6 ? 64 * (cB0 >> 2) : 0);
  const int prow_lim = (int)P.ldk;
  auto prefetch_macro = [&](int prow) {
    if (lane < G && prow < prow_lim) prefetch_l1(P.pool_comp + (size_t)prow * LPB + 128 * lane);
  };
  int pbase = 0;
  uint4 ca_n = ld_stream_v4(pa), cb_n = ld_stream_v4(pb);
  prefetch_macro(0);
#pragma unroll 1
  for (int mc = 0; mc < nmacro; ++mc) {
    const uint4 ca = ca_n, cb = cb_n;
    if (mc + 1 < nmacro) {
      ca_n = ld_stream_v4(pa + mc + 1);
      cb_n = ld_stream_v4(pb + mc + 1);
    }
    prefetch_macro(pbase + 8);
    const uint8_t *pcm = pc_thr + (size_t)pbase * LPB;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int s = j % NS;
      const uint8_t *pc = pcm + 128 * j;
      uint4 pcw[NBC];
#pragma unroll
      for (int i = 0; i < NBC; ++i) pcw[i] = __ldg(reinterpret_cast<const uint4 *>(pc) + i);
      const int codeA = LG == 6 ? code_of_rt(ca, j, shA) : code_of(ca, LG == 8 ? (j >> 1) : j);
      int k = (abs(codeA) * Lg) >> prec;
      if (LG == 8) k = (j & 1) ? max(k - 128, 0) : min(k, 128);
      const int kb = k - t0A;  // window end relative to this thread's first byte
      const uint32_t smA = (uint32_t)(codeA >> 31) | 0x01010101u;
      const int codeB = LG == 6 ? code_of_rt(cb, j, shB) : code_of(cb, LG == 8 ? (j >> 1) : j);
      const uint32_t u = (uint32_t)(abs(codeB) >> shift);
      const uint32_t smB = (uint32_t)(codeB >> 31) | 0x01010101u;
      const int kbmax = __reduce_max_sync(0xffffffffu, kb);
      const int kbmin = __reduce_min_sync(0xffffffffu, kb);
      if (!acquire_at(b, s, st.phase ^ (uint32_t)((j / NS) & 1))) return false;
      tc_fence_after();
      // ---- a: 16 words -> 16 TMEM columns of this lane
      uint32_t v[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (kbmax <= 16 * i) {  // warp-uniform: past every window
          v[4 * i] = v[4 * i + 1] = v[4 * i + 2] = v[4 * i + 3] = 0u;
        } else if (kbmin >= 16 * i + 16) {  // warp-uniform: inside every window
          v[4 * i] = v[4 * i + 1] = v[4 * i + 2] = v[4 * i + 3] = smA;
        } else {
          const uint32_t kc = (uint32_t)(kb - 16 * i);
          v[4 * i + 0] = prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x03020100u), 0u, 0xBA98u) & smA;
          v[4 * i + 1] = prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x07060504u), 0u, 0xBA98u) & smA;
          v[4 * i + 2] = prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x0B0A0908u), 0u, 0xBA98u) & smA;
          v[4 * i + 3] = prmt(mad_u32(kc, rep, 0x7F7F7F7Fu - 0x0F0E0D0Cu), 0u, 0xBA98u) & smA;
        }
      }
      tmem_st16(tA + (uint32_t)(s * Cfg::kAStageCols), v);
      // ---- b: streams into shared memory
      const uint32_t soff = (uint32_t)s * Cfg::kStageB;
#pragma unroll
      for (int i = 0; i < NBC; ++i) {
        st_shared_v4(sB[i] + soff,
                     prmt(mad_u32(u, rep, pcw[i].x), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].y), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].z), 0u, 0xBA98u) & smB,
                     prmt(mad_u32(u, rep, pcw[i].w), 0u, 0xBA98u) & smB);
      }
      // publish: b to the async proxy, the TMEM stores complete, then one
      // release per warp
      fence_async_smem();
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b.full[s]);
    }
    if ((G / NS) & 1) st.phase ^= 1u;
    pbase += 8;
  }
  return true;
}

// ---------------------------------------------------------------------------
// e2m1 operands.  {-1, 0, +1} are exact e2m1 values (nibbles 0xA, 0x0, 0x2),
// so with every block scale 1.0 the kind::mxf4 MMA computes the same bit
// products as kind::i8 at twice the elements per instruction: a 128-byte
// stage row carries 256 stream positions.  Nibble i (bits 4i .. 4i + 3) of
// word w of a row's k-block holds stream position 8 w + i; a and b use the
// same order, which is all the inner product needs.
//
//   a: positions t < k set: word = the sigma pattern (0x22222222 or
//      0xAAAAAAAA) cut to its low 4 (k - t0) - 32 w bits, one funnel shift
//      with the shift clamped to [0, 32];
//   b: [R[d'][t] < u] for the 8 positions of a word from two byte-SWAR
//      compares against a pool complement whose 8-byte groups hold positions
//      (0, 2, 4, 6 | 1, 3, 5, 7): even positions land in the low nibbles, odd
//      ones in the high nibbles, then the sigma pattern masks each nibble.
__device__ __forceinline__ uint32_t window_word_e2m1(uint32_t pattern, int k4, int w) {
  return __funnelshift_lc(pattern, 0u, (uint32_t)__viaddmax_s32(k4, -32 * w, 0));
}
__device__ __forceinline__ uint32_t stream_word_e2m1(uint32_t u, uint32_t rep, uint32_t pc_even,
                                                     uint32_t pc_odd, uint32_t pattern) {
  const uint32_t e = prmt(mad_u32(u, rep, pc_even), 0u, 0xBA98u);
  const uint32_t o = prmt(mad_u32(u, rep, pc_odd), 0u, 0xBA98u);
  return ((e & 0x0F0F0F0Fu) | (o & 0xF0F0F0F0u)) & pattern;
}

// Row producers of the e2m1 CTA pairs (Lp = 128 or 256; a stage = 256 stream
// positions of 256 a rows and `nb` b rows).  Thread pt owns a row pt % 256
// (bytes 64 (pt / 256) .. + 63, i.e. 128 positions: with Lp = 128 the whole
// stream of reduction index 2 j + pt / 256 of k-block j, with Lp = 256 the
// half pt / 256 of index j) and, for pt < 4 nb, b row pt % nb (bytes
// 32 (pt / nb) .. + 31: 64 positions).  Codes arrive 8 reduction indices per
// 16-byte load.
// kNoB: b arrives by TMA from a prepacked buffer; only the a rows are generated.
// kOneAcc: 128 a rows per CTA (one accumulator); thread pt owns a row pt % 128
// and its bytes 32 (pt / 128) .. + 31 (64 positions), like its b row.
// kSkipA: a 32-position chunk that lies past every window of the warp's 32
// rows is stored as zeros, one inside all of them as the sign pattern, both
// without arithmetic (exact; pays where windows are all short or all long,
// e.g. softmax rows in Attn@V).
// kSeg (one-accumulator pair tiles): K in segments of prm.kseg indices; the
// pool rows restart at every segment, and after each non-final segment the
// producers fold its counts into the running sums (segment_drain_pair, which
// needs tmem_base, warp and the tile's first b row n0_tile).
// mc_begin / mc_end: the macro steps (8 reduction indices each) of a K split
// (mc_end < 0: to the end of K).
template <int LG, int NS, bool kNoB, bool kOneAcc, bool kSkipA = false, bool kSeg = false>
__device__ bool produce_rows_fp4(const TcParams &prm, const Bars &b, ProdState &st,
                                 uint32_t smem_s, uint32_t stage_a_bytes, int lane, int64_t slice,
                                 int64_t slice_b, int64_t m0, int64_t n0, int nb,
                                 uint32_t tmem_base = 0, int warp = 0, int64_t n0_tile = 0,
                                 int mc_begin = 0, int mc_end = -1) {
  static_assert(LG == 7 || LG == 8, "e2m1 producers take Lp = 128 or 256");
  static_assert(!kSeg || kOneAcc, "segments run on one-accumulator tiles");
  if (!producers_released(b.abort)) return false;  // give-up path test hook
  constexpr int G = (8 << LG) / 256;  // k-blocks per macro step of 8 indices: 4 or 8
  constexpr int LPB = 1 << LG;
  constexpr int RA = kOneAcc ? 128 : 256;  // a rows per CTA
  constexpr int NCA = kOneAcc ? 2 : 4;     // a chunks (16 bytes) per thread
  // a macro step that is a whole number of ring turns starts at stage 0:
  // stage and phase of each k-block are then known at compile time
  constexpr bool kStatic = (G % NS) == 0;
  const GemmProblem &P = prm.P;
  const int pt = threadIdx.x - 32;
  const int ra = pt & (RA - 1);
  const int cA0 = NCA * (pt / RA);  // a chunks cA0 .. cA0 + NCA - 1
  const int hA = cA0 >> 2;          // Lp = 128: index 2 j + hA of k-block j
  // b: nb rows x 4 chunk pairs = 4 nb tasks over threads 0 .. 4 nb - 1, rows
  // fastest, so a narrow b side (Attn@V: 32 rows per CTA) is spread over
  // warps of all four SM sub-partitions instead of one
  const bool doB = pt < 4 * nb;
  const int rbn = doB ? pt % nb : 0;
  const int cB0 = doB ? 2 * (pt / nb) : 0;  // b chunks cB0, cB0 + 1
  const int64_t gmA = m0 + ra;
  const bool vA = gmA < prm.m_rows;
  const int64_t growA = slice * P.M + (vA ? gmA : prm.m_rows - 1);
  int Lg = 0;
  if (vA) {
    const int L = row_stream_len(P, slice, growA);
    Lg = L > 0 ? L : 0;
  }
  const int64_t gnB = n0 + rbn;
  const int64_t growB = slice_b * P.N + (gnB < prm.n_rows ? gnB : prm.n_rows - 1);
  const uint4 *pa = reinterpret_cast<const uint4 *>(P.qa.code + growA * P.ldk);
  const uint4 *pb = reinterpret_cast<const uint4 *>(P.qb.code + growB * P.ldk);
  uint32_t sA[NCA], sB[2];
#pragma unroll
  for (int i = 0; i < NCA; ++i) sA[i] = smem_s + sw128_offset(ra, cA0 + i);
#pragma unroll
  for (int i = 0; i < 2; ++i) sB[i] = smem_s + stage_a_bytes + sw128_offset(rbn, cB0 + i);
  // first position of this thread's a bytes inside its reduction index
  const int t0A = LG == 8 ? 32 * cA0 : 32 * (cA0 & 3);
  // Lp = 128: k-block j holds indices 2 j (bytes 0-63) and 2 j + 1 (64-127)
  const uint32_t shA = 16u - 16u * (uint32_t)hA;
  const uint32_t shB = 16u - 16u * (uint32_t)(cB0 >> 2);
  const uint32_t rep = prm.rep;
  const int prec = P.prec;
  const int shift = prm.shift_pool;
  const int nmacro = mc_end < 0 ? (int)(P.ldk >> 3) : mc_end;
  // pool complement: k-block j of a macro step starts 256 bytes after j - 1;
  // this thread's 64 positions are 64 bytes at 32 cB0 into it
  const uint8_t *pc_thr = P.pool_comp + 32 * cB0;
  const int prow_lim = (int)P.ldk;
  auto prefetch_macro = [&](int prow) {
    if (lane < LPB / 16 && prow < prow_lim)
      prefetch_l1(P.pool_comp + (size_t)prow * LPB + 128 * lane);
  };
  int pbase = 8 * mc_begin;  // pool row of the macro step's first reduction index
  const int msteps_seg = kSeg ? prm.kseg >> 3 : 0;  // macro steps per segment
  int mseg = 0;                                     // macro steps done in the segment
  uint4 ca_n = ld_stream_v4(pa + mc_begin), cb_n = make_uint4(0, 0, 0, 0);
  // One-accumulator tiles (8 a words per thread) have the registers to load
  // the next stage's pool complement words one stage ahead, keeping their
  // latency off each stage's acquire -> store -> publish chain; the others
  // load them at the top of the stage.
  // (Segmented tiles leave those 16 registers to the segment drain: 17 warps
  // give each thread at most 96.)
  constexpr bool kAheadPC = kOneAcc && !kSeg;
  uint4 qn0 = make_uint4(0, 0, 0, 0), qn1 = qn0, qn2 = qn0, qn3 = qn0;
  if constexpr (!kNoB) {
    if (doB) {
      cb_n = ld_stream_v4(pb + mc_begin);
      if constexpr (kAheadPC) {
        const uint4 *pc = reinterpret_cast<const uint4 *>(pc_thr + (size_t)pbase * LPB);
        qn0 = __ldg(pc);
        qn1 = __ldg(pc + 1);
        qn2 = __ldg(pc + 2);
        qn3 = __ldg(pc + 3);
      }
    }
    prefetch_macro(pbase);
  }
#pragma unroll 1
  for (int mc = mc_begin; mc < nmacro; ++mc) {
    const uint4 ca = ca_n, cb = cb_n;
    if (mc + 1 < nmacro) {
      ca_n = ld_stream_v4(pa + mc + 1);
      if (!kNoB && doB) cb_n = ld_stream_v4(pb + mc + 1);
    }
    const bool seg_end = kSeg && mseg + 1 == msteps_seg;  // the next step starts a segment
    if constexpr (!kNoB) prefetch_macro(seg_end ? 0 : pbase + 8);
    const uint8_t *pcm = pc_thr + (size_t)pbase * LPB;
    // pool rows of the next macro step: 8 rows on, or row 0 of a new segment
    const uint8_t *pcm_next = seg_end ? pc_thr : pcm + 256 * G;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      uint4 q0 = qn0, q1 = qn1, q2 = qn2, q3 = qn3;
      if (kAheadPC && !kNoB && doB && (j + 1 < G || mc + 1 < nmacro)) {
        // stage j + 1 of this macro step, or stage 0 of the next one
        const uint4 *pc = reinterpret_cast<const uint4 *>(j + 1 < G ? pcm + 256 * (j + 1)
                                                                    : pcm_next);
        qn0 = __ldg(pc);
        qn1 = __ldg(pc + 1);
        qn2 = __ldg(pc + 2);
        qn3 = __ldg(pc + 3);
      }
      if (!kAheadPC && !kNoB && doB) {
        const uint4 *pc = reinterpret_cast<const uint4 *>(pcm + 256 * j);
        q0 = __ldg(pc);
        q1 = __ldg(pc + 1);
        q2 = __ldg(pc + 2);
        q3 = __ldg(pc + 3);
      }
      const int codeA = LG == 7 ? code_of_rt(ca, j, shA) : code_of(ca, j);
      const int k = (abs(codeA) * Lg) >> prec;
      const int k4 = 4 * (k - t0A);
      const uint32_t patA = codeA < 0 ? 0xAAAAAAAAu : 0x22222222u;
      const int codeB = LG == 7 ? code_of_rt(cb, j, shB) : code_of(cb, j);
      const uint32_t u = (uint32_t)(abs(codeB) >> shift);
      const uint32_t patB = codeB < 0 ? 0xAAAAAAAAu : 0x22222222u;
      uint32_t soff;
      if constexpr (kStatic) {
        if (!acquire_at(b, j % NS, st.phase ^ (uint32_t)((j / NS) & 1))) return false;
        soff = (uint32_t)(j % NS) * prm.stage_bytes;
      } else {
        if (!acquire_stage(b, st, lane)) return false;
        soff = mad_u32((uint32_t)st.stage, prm.stage_bytes, 0u);
      }
      // window end relative to this thread's first position, over the warp
      const int relmax = kSkipA ? __reduce_max_sync(0xffffffffu, k - t0A) : 0;
      const int relmin = kSkipA ? __reduce_min_sync(0xffffffffu, k - t0A) : 0;
#pragma unroll
      for (int i = 0; i < NCA; ++i) {
        if (kSkipA && relmax <= 32 * i) {  // warp-uniform: past every window
          st_shared_v4(sA[i] + soff, 0u, 0u, 0u, 0u);
        } else if (kSkipA && relmin >= 32 * i + 32) {  // warp-uniform: inside every window
          st_shared_v4(sA[i] + soff, patA, patA, patA, patA);
        } else {
          st_shared_v4(sA[i] + soff, window_word_e2m1(patA, k4, 4 * i),
                       window_word_e2m1(patA, k4, 4 * i + 1),
                       window_word_e2m1(patA, k4, 4 * i + 2),
                       window_word_e2m1(patA, k4, 4 * i + 3));
        }
      }
      if (!kNoB && doB) {
        st_shared_v4(sB[0] + soff, stream_word_e2m1(u, rep, q0.x, q0.y, patB),
                     stream_word_e2m1(u, rep, q0.z, q0.w, patB),
                     stream_word_e2m1(u, rep, q1.x, q1.y, patB),
                     stream_word_e2m1(u, rep, q1.z, q1.w, patB));
        st_shared_v4(sB[1] + soff, stream_word_e2m1(u, rep, q2.x, q2.y, patB),
                     stream_word_e2m1(u, rep, q2.z, q2.w, patB),
                     stream_word_e2m1(u, rep, q3.x, q3.y, patB),
                     stream_word_e2m1(u, rep, q3.z, q3.w, patB));
      }
      if constexpr (kStatic)
        publish_at(b, j % NS, lane);
      else
        publish_stage<NS>(b, st, lane);
    }
    if constexpr (kStatic) {
      if ((G / NS) & 1) st.phase ^= 1u;
    }
    pbase += 8;
    if constexpr (kSeg) {
      if (++mseg == msteps_seg) {
        mseg = 0;
        pbase = 0;
        // ---- end of a segment (the last one drains in the epilogue)
        if (mc + 1 < nmacro &&
            !segment_drain_pair(prm, b, st, tmem_base, warp, lane, (mc + 1) / msteps_seg - 1,
                                slice, slice_b, m0, n0_tile))
          return false;
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Epilogue: TMEM -> smem transpose -> rescale -> bias -> coalesced stores.
// The stage ring is idle (every MMA of this tile has completed), so each warp
// stages its 32x32 blocks there; a producer-only barrier keeps the next
// tile's operand writes out until all are done.
// kF32: the accumulators hold fp32 counts (e2m1 pairs: exact integers, see
// gemm_tc_pair_fp4_kernel) in two blocks of prm.ncols columns; columns past
// prm.ncols are not part of the tile.  kOneAcc: one accumulator of 128 a rows
// (lanes) x prm.ncols columns; warp pw takes the 32-column chunks pw / 4,
// pw / 4 + 4, ...
// part != NULL (a K split): store the tile's exact int32 counts there
// ([batch, M, N] layout) instead of rescaled outputs.
template <int BN, bool kSeg, bool kPair = false, bool kF32 = false, bool kOneAcc = false>
__device__ bool tile_epilogue(const TcParams &prm, const Bars &b, ProdState &st,
                              unsigned char *smem, uint32_t tmem_base, int warp, int lane,
                              int64_t slice, int64_t slice_b, int64_t m0, int64_t n0, int64_t it,
                              int32_t *part = nullptr) {
  static_assert(!kOneAcc || kF32, "one-accumulator tiles are e2m1 pair tiles");
  const GemmProblem &P = prm.P;
  const int ncols = kF32 ? prm.ncols : BN;
  if (!mbar_wait(b.tfull, (uint32_t)(st.g & 1), b.abort)) return false;
  tc_fence_after();
  {
    const int pw = warp - 1;                 // producer warp 0..15
    const int quarter = warp & 3;            // TMEM lanes this warp may access
    const int acc_j = kOneAcc ? 0 : (pw >> 2) & 1;  // accumulator (a rows 0-127 / 128-255)
    const int col_half = pw >> 3;            // which half of the BN columns
    // two accumulators: each column half takes ceil(ncols / 64) 32-column
    // chunks (BN / 64 of them on the int8 tiles)
    const int per_half = kF32 ? (ncols + 63) / 64 : BN / 64;
    const int cc_begin = kOneAcc ? (pw >> 2) : col_half * per_half;
    const int cc_end = kOneAcc ? (ncols + 31) / 32 : (col_half + 1) * per_half;
    const int cc_step = kOneAcc ? 4 : 1;
    float *stg = reinterpret_cast<float *>(smem) + pw * (32 * 33);
    int4 *rowp = reinterpret_cast<int4 *>(smem + kProducerWarps * 32 * 33 * 4) + pw * 32;
    float *rowF = reinterpret_cast<float *>(smem + kProducerWarps * 32 * 33 * 4 +
                                            kProducerWarps * 32 * 16) + pw * 32;
    const int64_t mrow0 = m0 + acc_j * 128 + quarter * 32;  // first row of this warp
    {
      const int64_t gm = mrow0 + lane;
      int L = -1, za = 0, rsa = 0;
      float sa = 0.f;
      if (gm < prm.m_rows) {
        const int64_t grow = slice * P.M + gm;
        L = row_stream_len(P, slice, grow);
        sa = P.qa.scale[grow];
        za = P.qa.zero[grow];
        rsa = P.qa.rowsum[grow];
      }
      rowp[lane] = make_int4(L, __float_as_int(sa), za, rsa);
      rowF[lane] = L > 0 ? sc_rescale_factor(P.mode, P.prec, L) : 0.0f;
    }
    __syncwarp();
    const int64_t grow0 = slice * P.M + mrow0;
    const int myL = rowp[lane].x;  // stream length of this lane's row
    // Bipolar outputs without counts to keep: the rescale ((acc * sa) * (sb *
    // F), the oracle's order) is split at its first product, taken while a
    // lane holds a row; after the transpose each element costs two multiplies.
    const bool fast = !kSeg && P.mode == SCMP_BIPOLAR && part == nullptr && P.acc_out == nullptr;
    const uint32_t skip_rows = __ballot_sync(0xffffffffu, myL < 0);  // rows of another call
#pragma unroll 1
    for (int cc = cc_begin; cc < cc_end; cc += cc_step) {
      if (kF32 && cc * 32 >= ncols) break;  // warp-uniform
      if constexpr (kSeg && kF32) {
        // last segment of an e2m1 tile: accumulator acc_j's counts in columns
        // acc_j ncols + c, its running sums (kOneAcc ? 1 : 2) ncols further on
        const uint32_t acc0 = (uint32_t)(acc_j * ncols);
        const uint32_t run0 = (uint32_t)((kOneAcc ? 1 : 2) * ncols) + acc0;
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {
          const int c = cc * 32 + h * 8;
          uint32_t v[8];
          if (c < ncols) {
            seg_chunk16<true, 8>(prm, tmem_base + ((uint32_t)(quarter * 32) << 16), lane,
                                 prm.nseg - 1, acc0 + (uint32_t)c, run0 + (uint32_t)c, n0 + c,
                                 grow0 + lane, mrow0 + lane < prm.m_rows, myL, slice_b, v);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0u;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) stg[lane * 33 + h * 8 + i] = __uint_as_float(v[i]);
        }
      } else if constexpr (kSeg) {
        // last segment: finished fp32 values (rescaled and summed in order)
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t v[16];
          seg_chunk<BN>(prm, tmem_base, lane, prm.nseg - 1, cc, h, acc_j, quarter, grow0 + lane,
                        mrow0 + lane < prm.m_rows, myL, slice_b, n0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) stg[lane * 33 + h * 16 + i] = __uint_as_float(v[i]);
        }
      } else {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc_j * ncols + cc * 32),
                  v);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (fast) {
          // count * sa of this lane's row (pruned rows: 0); e2m1 counts are
          // exact integers in fp32, so (float)acc is the loaded value
          const float sa_l = myL > 0 ? __int_as_float(rowp[lane].y) : 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float cnt = kF32 ? __uint_as_float(v[i]) : (float)(int32_t)v[i];
            stg[lane * 33 + i] = myL > 0 ? __fmul_rn(cnt, sa_l) : 0.0f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)  // int32 counts as their bit patterns
            stg[lane * 33 + i] = kF32 ? __int_as_float(__float2int_rn(__uint_as_float(v[i])))
                                      : __uint_as_float(v[i]);
        }
      }
      __syncwarp();
      // lane = column now
      const int64_t gn = n0 + cc * 32 + lane;
      const bool col_ok = gn < prm.n_rows && (!kF32 || cc * 32 + lane < ncols);
      float sb = 0.f;
      int32_t zb = 0, rsb = 0;
      float bias = 0.f;
      if (col_ok) {
        const int64_t brw = slice_b * P.N + gn;
        sb = P.qb.scale[brw];
        zb = P.qb.zero[brw];
        rsb = P.qb.rowsum[brw];
        if (P.bias) bias = P.bias[gn];
      }
      if (!kSeg && fast) {
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
          if ((skip_rows >> r) & 1u) continue;  // warp-uniform
          // sb * F (F = 0 on pruned rows), then (count * sa) * that
          const float fb = __fmul_rn(sb, rowF[r]);
          float y = __fmul_rn(stg[r * 33 + lane], fb);
          if (P.bias) y = __fadd_rn(y, bias);
          if (col_ok) store_out(P, (grow0 + r) * P.N + gn, y);
        }
        __syncwarp();
        continue;
      }
#pragma unroll 4
      for (int r = 0; r < 32; ++r) {
        const int4 rp = rowp[r];  // broadcast
        if (!col_ok || rp.x < 0) continue;
        const int32_t a = rp.x > 0 ? __float_as_int(stg[r * 33 + lane]) : 0;
        if (!kSeg && part) {
          part[(grow0 + r) * P.N + gn] = a;
          continue;
        }
        float y = 0.0f;
        if constexpr (kSeg) {
          if (rp.x > 0) y = stg[r * 33 + lane];
        } else if (rp.x > 0) {
          y = sc_rescale_f(P.mode, rowF[r], a, P.K, __int_as_float(rp.y), rp.z, rp.w, sb, zb,
                         rsb);
        }
        if (P.bias) y = __fadd_rn(y, bias);
        const int64_t o = (grow0 + r) * P.N + gn;
        store_out(P, o, y);
        if (!kSeg && P.acc_out) P.acc_out[o] = a;
      }
      __syncwarp();
    }
  }
  // every producer is done with the staging area before anyone refills it
  // (a bounded mbarrier wait, not bar.sync: an aborting thread must not
  // leave the others blocked)
  // On CTA pairs the epi barrier completes once per (tile, segment) --
  // segment_drain_pair uses it too -- so its phase is that of st.g (= it when
  // unsegmented); single-CTA tiles use it once per tile.
  if constexpr (kPair) {
    // one thread per CTA hands the accumulators back to the even CTA's MMA
    // thread once every producer of this CTA has read them
    tc_fence_before();
    mbar_arrive(b.epi);
    if (!mbar_wait(b.epi, (uint32_t)(st.g & 1), b.abort)) return false;
    if (threadIdx.x == 32) mbar_arrive_cluster(b.tempty_cl);
  } else {
    mbar_arrive(b.epi);
    if (!mbar_wait(b.epi, (uint32_t)(it & 1), b.abort)) return false;
    tc_fence_before();
    mbar_arrive(b.tempty);
  }
  ++st.g;
  return true;
}

template <int BN, int kProd, int LG, bool kSeg>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const TcParams prm) {
  using Cfg = TcCfg<BN>;
  // int32 accumulators in columns [0, 2 BN); segmented kernels keep the fp32
  // running sum of the finished segments in columns [2 BN, 4 BN)
  constexpr uint32_t kTmemAlloc = kSeg ? 4 * BN : 2 * BN;
  static_assert(!kSeg || BN <= 128, "segmented tiles need 4*BN <= 512 TMEM columns");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *therm_s = smem + Cfg::kNS * Cfg::kStage;  // [sign][window 0..128][128 B]
  Bars b;
  b.full = reinterpret_cast<uint64_t *>(therm_s + (kProd == kProdTable ? Cfg::kTherm : 0));
  b.empty = b.full + Cfg::kNS;
  b.tfull = b.empty + Cfg::kNS;
  b.tempty = b.tfull + 1;
  b.drain = b.tempty + 1;
  b.epi = b.drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(b.epi + 1);
  b.abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kNS; ++s) {
      mbar_init(&b.full[s], kProducerWarps);
      mbar_init(&b.empty[s], 1);
    }
    mbar_init(b.tfull, 1);
    mbar_init(b.tempty, kProducers);
    mbar_init(b.drain, 1);
    mbar_init(b.epi, kProducers);
    *b.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if constexpr (kProd == kProdTable) {
    const uint4 *src = reinterpret_cast<const uint4 *>(prm.therm);
    uint4 *dst = reinterpret_cast<uint4 *>(therm_s);
    for (int i = threadIdx.x; i < (int)(Cfg::kTherm / 16); i += blockDim.x) dst[i] = __ldg(src + i);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ================================================= MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8<BN>();
      const uint32_t smem0 = smem_u32(smem);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t g = 0;  // drain counter: one per (tile, segment)
      for (int64_t tile = blockIdx.x; tile < prm.tiles && ok; tile += gridDim.x) {
        for (int seg = 0; seg < prm.nseg && ok; ++seg, ++g) {
          // the accumulators are free once the previous drain has read them
          if (g > 0) ok = mbar_wait(b.tempty, (uint32_t)((g - 1) & 1), b.abort);
          if (!ok) break;
          tc_fence_after();
          for (int64_t kb = 0; kb < prm.nkb_seg; ++kb) {
            if (!mbar_wait(&b.full[stage], phase, b.abort)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a0 = smem0 + stage * Cfg::kStage;
            const uint32_t b0 = a0 + Cfg::kStageA;
#pragma unroll
            for (int kk = 0; kk < kKB / 32; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(b0 + kk * 32);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const uint64_t adesc = smem_desc_sw128(a0 + j * (128 * kKB) + kk * 32);
                tc_mma_i8(tmem_base + j * BN, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              }
            }
            tc_commit(&b.empty[stage]);
            if (++stage == Cfg::kNS) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          tc_commit(b.tfull);
        }
      }
      // Drain: everything this thread issued has completed before TMEM is freed.
      tc_commit(b.drain);
      mbar_wait_own(b.drain, 0);
    }
    __syncwarp();
  } else {
    // ============================ producers + epilogue (kProducerWarps warps)
    const uint32_t smem_s = smem_u32(smem);  // 32-bit shared-window addresses
    const uint32_t therm_u = smem_u32(therm_s);
    ProdState st{0, 0u, 0};
    int64_t it = 0;
    for (int64_t tile = blockIdx.x; tile < prm.tiles; tile += gridDim.x, ++it) {
      const int64_t slice = tile / (prm.tiles_m * prm.tiles_n);
      const int64_t rem = tile % (prm.tiles_m * prm.tiles_n);
      const int64_t m0 = (rem % prm.tiles_m) * kBM;
      const int64_t n0 = (rem / prm.tiles_m) * BN;
      const int64_t slice_b = prm.P.batch_b == 1 ? 0 : slice;
      bool ok;
      if constexpr (kProd == kProdRows)
        ok = produce_rows<BN, LG, kSeg, Cfg::kNS, false, false, BN == 64>(
            prm, b, st, smem_s, tmem_base, warp, lane, slice, slice_b,
                                        m0, n0);
      else
        ok = produce_chunks<BN, kProd == kProdTable, kSeg>(prm, b, st, smem_s, therm_u, tmem_base,
                                                           warp, lane, slice, slice_b, m0, n0);
      if (!ok) break;
      if (!tile_epilogue<BN, kSeg>(prm, b, st, smem, tmem_base, warp, lane, slice, slice_b, m0, n0,
                                   it))
        break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
  }
  if (threadIdx.x == 0 && *b.abort) atomicOr(prm.error, 1u);
}

// Narrow-tile kernel with the window operand in TMEM (unsegmented row
// producers, BN <= 128): warp 0 issues M = 128 x N = BN MMAs whose A is a TMEM
// stage and whose B is a shared-memory stage; warps 1..16 generate both and
// run the epilogue.  The whole TMEM (512 columns) is allocated: one CTA per SM.
template <int BN, int LG>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_ts_kernel(const TcParams prm) {
  using Cfg = TsCfg<BN>;
  constexpr uint32_t kTmemAlloc = 512;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars b;
  b.full = reinterpret_cast<uint64_t *>(smem + Cfg::kRing);
  b.empty = b.full + kTsStages;
  b.tfull = b.empty + kTsStages;
  b.tempty = b.tfull + 1;
  b.drain = b.tempty + 1;
  b.epi = b.drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(b.epi + 1);
  b.abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTsStages; ++s) {
      mbar_init(&b.full[s], kProducerWarps);
      mbar_init(&b.empty[s], 1);
    }
    mbar_init(b.tfull, 1);
    mbar_init(b.tempty, kProducers);
    mbar_init(b.drain, 1);
    mbar_init(b.epi, kProducers);
    *b.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ================================================= MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8<BN>();
      const uint32_t smem0 = smem_u32(smem);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t g = 0;
      for (int64_t tile = blockIdx.x; tile < prm.tiles && ok; tile += gridDim.x, ++g) {
        if (g > 0) ok = mbar_wait(b.tempty, (uint32_t)((g - 1) & 1), b.abort);
        if (!ok) break;
        tc_fence_after();
        for (int64_t kb = 0; kb < prm.nkb; ++kb) {
          if (!mbar_wait(&b.full[stage], phase, b.abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t b0 = smem0 + stage * Cfg::kStageB;
          const uint32_t a0 = tmem_base + Cfg::kAcol + (uint32_t)stage * Cfg::kAStageCols;
#pragma unroll
          for (int kk = 0; kk < kKB / 32; ++kk) {
            const uint64_t bdesc = smem_desc_sw128(b0 + kk * 32);
#pragma unroll
            for (int j = 0; j < 2; ++j)  // 32 bytes of K = 8 columns
              tc_mma_i8_ts(tmem_base + j * BN, a0 + (uint32_t)(j * 32 + kk * 8), bdesc, idesc,
                           (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&b.empty[stage]);
          if (++stage == kTsStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(b.tfull);
      }
      // Drain: everything this thread issued has completed before TMEM is freed.
      tc_commit(b.drain);
      mbar_wait_own(b.drain, 0);
    }
    __syncwarp();
  } else {
    // ============================ producers + epilogue (kProducerWarps warps)
    const uint32_t smem_s = smem_u32(smem);
    ProdState st{0, 0u, 0};
    int64_t it = 0;
    for (int64_t tile = blockIdx.x; tile < prm.tiles; tile += gridDim.x, ++it) {
      const int64_t slice = tile / (prm.tiles_m * prm.tiles_n);
      const int64_t rem = tile % (prm.tiles_m * prm.tiles_n);
      const int64_t m0 = (rem % prm.tiles_m) * kBM;
      const int64_t n0 = (rem / prm.tiles_m) * BN;
      const int64_t slice_b = prm.P.batch_b == 1 ? 0 : slice;
      if (!produce_rows_ts<BN, LG>(prm, b, st, smem_s, tmem_base, warp, lane, slice, slice_b, m0,
                                   n0))
        break;
      if (!tile_epilogue<BN, false>(prm, b, st, smem, tmem_base, warp, lane, slice, slice_b, m0,
                                    n0, it))
        break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
  }
  if (threadIdx.x == 0 && *b.abort) atomicOr(prm.error, 1u);
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (cta_group::2; unsegmented row producers, N >= 129).
// A 2-CTA cluster owns a 512 x 256 output tile: CTA q generates a rows
// m0 + 256 q .. + 255 and b rows n0 + 128 q .. + 127 of every k-block; the
// even CTA issues M = 256 x N = 256 MMAs that read both CTAs' shared memory,
// and each CTA's TMEM receives its own 256 a rows x all 256 columns.  Per
// CTA this generates 384 operand rows per k-block instead of 512 and reads
// 64 KB of shared memory per k-block for the MMAs instead of 96 KB; a stage
// is 48 KB, so four fit.
constexpr int kPairStages = 4;
constexpr uint32_t kPairStageA = kBM * kKB;          // 32 KB: 256 a rows
constexpr uint32_t kPairStageB = 128 * kKB;          // 16 KB: this CTA's 128 b rows
constexpr uint32_t kPairStage = kPairStageA + kPairStageB;
static_assert(kPairStage == TcCfg<128>::kStage, "pair producers use the BN = 128 stage layout");
constexpr size_t kPairSmem = (size_t)kPairStages * kPairStage + 1024 /*align*/ + 256;

// Instruction descriptor for the pair MMA: s8 x s8 -> s32, K-major, M = 256, N = 256.
constexpr uint32_t kIdescPair = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                                ((uint32_t)(256 >> 4) << 24);

// With kPackedB the b halves come from a prepacked buffer by TMA: warp
// kTmaWarp (an 18th warp) loads this CTA's 128 b rows of each k-block and the
// producers generate only the a rows.
constexpr int kTmaWarp = 1 + kProducerWarps;
constexpr int kL2Ahead = 16;  // k-blocks between a b tile's L2 prefetch and its load

template <int LG, bool kPackedB>
__global__ void __launch_bounds__(kThreads + 32, 1)
    gemm_tc_pair_kernel(const TcParams prm, const __grid_constant__ CUtensorMap tmap) {
  constexpr uint32_t kTmemAlloc = 512;  // two 256-column accumulators
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars b;
  b.full = reinterpret_cast<uint64_t *>(smem + kPairStages * kPairStage);
  b.empty = b.full + kPairStages;
  b.pfull = b.empty + kPairStages;
  b.tfull = b.pfull + kPairStages;
  b.tempty = b.tfull + 1;
  b.drain = b.tempty + 1;
  b.epi = b.drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(b.epi + 1);
  b.abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      // this CTA's producer warps (+ the TMA thread's expect_tx arrival)
      mbar_init(&b.full[s], kProducerWarps + (kPackedB ? 1 : 0));
      mbar_init(&b.empty[s], 1);
      mbar_init(&b.pfull[s], 1);              // the odd CTA's stage (even CTA only)
    }
    mbar_init(b.tfull, 1);
    mbar_init(b.tempty, 2);  // one arrival per CTA after its epilogue
    mbar_init(b.drain, 1);
    mbar_init(b.epi, kProducers);
    *b.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone arrives on them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  b.pfull_cl = mapa_shared(smem_u32(b.pfull), 0);
  b.tempty_cl = mapa_shared(smem_u32(b.tempty), 0);
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t nclusters = gridDim.x >> 1;

  if (warp == 0) {
    // ====================================== MMA issuer (even CTA, lane 0)
    if (rank == 0 && lane == 0) {
      const uint32_t smem0 = smem_u32(smem);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t g = 0;  // tiles issued
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters, ++g) {
        // both CTAs have read the previous tile's accumulators
        if (g > 0) ok = mbar_wait_cl(b.tempty, (uint32_t)((g - 1) & 1), b.abort);
        if (!ok) break;
        tc_fence_after();
        for (int64_t kb = 0; kb < prm.nkb; ++kb) {
          // this CTA's stage, then the odd CTA's (forwarded at cluster scope)
          if (!mbar_wait(&b.full[stage], phase, b.abort) ||
              !mbar_wait_cl(&b.pfull[stage], phase, b.abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem0 + stage * kPairStage;
          const uint32_t b0 = a0 + kPairStageA;
#pragma unroll
          for (int kk = 0; kk < kKB / 32; ++kk) {
            const uint64_t bdesc = smem_desc_sw128(b0 + kk * 32);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint64_t adesc = smem_desc_sw128(a0 + j * (128 * kKB) + kk * 32);
              tc_mma_i8_pair(tmem_base + j * 256, adesc, bdesc, kIdescPair,
                             (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc_commit_pair_both(&b.empty[stage]);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair_both(b.tfull);
      }
      // Drain: everything this thread issued has completed before TMEM is freed.
      tc_commit_pair_local(b.drain);
      mbar_wait_own_cl(b.drain, 0);
    } else if (rank == 1 && lane == 0) {
      // ============ forwarder (odd CTA): each filled stage of this CTA is
      // announced to the MMA thread with one cluster-scope release
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters) {
        for (int64_t kb = 0; kb < prm.nkb; ++kb) {
          if (!mbar_wait(&b.full[stage], phase, b.abort)) { ok = false; break; }
          mbar_arrive_cluster(b.pfull_cl + 8u * (uint32_t)stage);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (kPackedB && warp == kTmaWarp) {
    // ========================== b loader (lane 0): prepacked rows by TMA
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      const uint32_t smem0 = smem_u32(smem);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t it = 0;
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters, ++it) {
        const int64_t rem = tile % (prm.tiles_m * prm.tiles_n);
        const int nb0 = (int)((rem / prm.tiles_m) * 256 + (int64_t)rank * 128);
        // the previous tile's epilogue stages its transpose in the ring
        if (it > 0 && !mbar_wait(b.epi, (uint32_t)((it - 1) & 1), b.abort)) break;
        for (int64_t kb = 0; kb < prm.nkb; ++kb) {
          if (!mbar_wait(&b.empty[stage], phase ^ 1, b.abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&b.full[stage], kPairStageB);
          tma_load_2d(smem0 + stage * kPairStage + kPairStageA, &tmap, (int)(kb * kKB), nb0,
                      &b.full[stage]);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else {
    // ============================ producers + epilogue (kProducerWarps warps)
    const uint32_t smem_s = smem_u32(smem);
    ProdState st{0, 0u, 0};
    int64_t it = 0;
    for (int64_t tile = cluster; tile < prm.tiles; tile += nclusters, ++it) {
      const int64_t slice = tile / (prm.tiles_m * prm.tiles_n);
      const int64_t rem = tile % (prm.tiles_m * prm.tiles_n);
      const int64_t m0 = (rem % prm.tiles_m) * (2 * kBM) + (int64_t)rank * kBM;
      const int64_t n0 = (rem / prm.tiles_m) * 256;
      const int64_t slice_b = prm.P.batch_b == 1 ? 0 : slice;
      if (!produce_rows<128, LG, false, kPairStages, true, kPackedB>(
              prm, b, st, smem_s, tmem_base, warp, lane, slice, slice_b, m0,
              n0 + (int64_t)rank * 128))
        break;
      if (!tile_epilogue<256, false, true>(prm, b, st, smem, tmem_base, warp, lane, slice, slice_b,
                                           m0, n0, it))
        break;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while the pair may still touch its memory
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
  }
  if (threadIdx.x == 0 && *b.abort) atomicOr(prm.error, 1u);
}

// ---------------------------------------------------------------------------
// CTA pairs on e2m1 operands (tcgen05.mma kind::mxf4, block32 scales all 1.0).
// Same cluster protocol, stage ring and epilogue as gemm_tc_pair_kernel; a
// stage carries 256 stream positions, the tile is 512 a rows x prm.ncols b
// rows (ncols <= 240, a multiple of 16: CTA q generates b rows
// n0 + q ncols / 2 ..), and TMEM holds the two fp32 accumulators in columns
// [0, 2 ncols) and the E8M0 scale factors (0x7F = 1.0 in every byte) in
// columns [kFp4SfCol, 512).  Counts stay exact while K * Lp < 2^24.
constexpr uint32_t kFp4SfCol = 480;
constexpr int kFp4MaxCols = 240;
static_assert(2 * kFp4MaxCols <= (int)kFp4SfCol, "accumulators below the scale factors");

__host__ __device__ constexpr uint32_t idesc_mxf4_pair(int n) {
  return (1u << 7)                       // A format E2M1
         | (1u << 10)                    // B format E2M1
         | ((uint32_t)(n >> 3) << 17)    // N >> 3
         | (1u << 23)                    // scale factors E8M0
         | ((uint32_t)(256 >> 4) << 24);  // M = 256 (two CTAs); K = 64
}
__device__ __forceinline__ void tc_mma_mxf4_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t tmem_sfa,
                                                 uint32_t tmem_sfb, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], "
      "p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tmem_sfa), "r"(tmem_sfb)
      : "memory");
}

// With kPackedB the b halves come from a prepacked e2m1 buffer by TMA: warp
// kTmaWarp loads this CTA's ncols / 2 b rows of each stage and the producers
// generate only the a rows.
//
// kOneAcc: 256-row tiles (128 a rows per CTA, one accumulator of ncols <= 256
// columns, M = 256 MMAs once per 64 positions); stages are 32 KB.  Taken when
// one 512-row tile would be half empty or the b side is narrow (Q@K^T and
// Attn@V per head: 256 x 256 and 256 x 64).
template <bool kOneAcc, int kNStages = kPairStages>
struct Fp4PairCfg {
  static constexpr uint32_t kStageA = (kOneAcc ? 128 : 256) * kKB;
  static constexpr uint32_t kStage = kStageA + kPairStageB;
  // four stages (six 32 KB stages measured no faster on Q@K^T or on the
  // segmented compensation tiles)
  static constexpr int kStages = kNStages;
  static constexpr size_t kSmem = (size_t)kStages * kStage + 1024 /*align*/ + 256;
  static_assert(kStages * kStage >= kEpiStagingBytes, "the ring holds the epilogue staging");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};
// Ring depth of the segmented one-accumulator tiles (six measured no faster
// on the compensation shape than four).
constexpr int kSegPairStages = 4;

// kSeg (one accumulator): K in prm.nseg segments of prm.nkb_seg k-blocks; the
// MMA thread restarts the accumulator at every segment and waits for the
// producers' drain of the previous one (tempty); the fp32 running sums live in
// TMEM columns [ncols, 2 ncols) (ncols <= 240).  Two accumulators would leave
// room for 112 columns only and measured slower on the compensation shape.
// kSplit: the tiles of prm.ksplit K splits (see TcParams), counts to prm.part.
template <int LG, bool kPackedB, bool kOneAcc, bool kSeg = false, bool kSplit = false>
__global__ void __launch_bounds__(kThreads + 32, 1)
    gemm_tc_pair_fp4_kernel(const TcParams prm, const __grid_constant__ CUtensorMap tmap) {
  static_assert(!(kSeg && kSplit), "segmented K is not split");
  static_assert(!kSeg || kOneAcc, "segments run on one-accumulator tiles");
  using Cfg = Fp4PairCfg<kOneAcc, kSeg ? kSegPairStages : kPairStages>;
  constexpr uint32_t kTmemAlloc = 512;
  constexpr int kAcc = kOneAcc ? 1 : 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars b;
  b.full = reinterpret_cast<uint64_t *>(smem + Cfg::kStages * Cfg::kStage);
  b.empty = b.full + Cfg::kStages;
  b.pfull = b.empty + Cfg::kStages;
  b.tfull = b.pfull + Cfg::kStages;
  b.tempty = b.tfull + 1;
  b.drain = b.tempty + 1;
  b.epi = b.drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(b.epi + 1);
  b.abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int ncols = prm.ncols;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      // this CTA's producer warps (+ the TMA thread's expect_tx arrival)
      mbar_init(&b.full[s], kProducerWarps + (kPackedB ? 1 : 0));
      mbar_init(&b.empty[s], 1);
      mbar_init(&b.pfull[s], 1);
    }
    mbar_init(b.tfull, 1);
    mbar_init(b.tempty, 2);
    mbar_init(b.drain, 1);
    mbar_init(b.epi, kProducers);
    *b.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // unit scale factors in this CTA's columns [kFp4SfCol, 512), every lane
  // (warps 1-4 cover the four lane quarters)
  if (warp >= 1 && warp <= 4) {
    uint32_t one[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) one[i] = 0x7F7F7F7Fu;
    const uint32_t t = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + kFp4SfCol;
    tmem_st16(t, one);
    tmem_st16(t + 16, one);
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers and scale factors exist before any MMA
  tc_fence_after();
  b.pfull_cl = mapa_shared(smem_u32(b.pfull), 0);
  b.tempty_cl = mapa_shared(smem_u32(b.tempty), 0);
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t nclusters = gridDim.x >> 1;

  if (warp == 0) {
    // ====================================== MMA issuer (even CTA, lane 0)
    if (rank == 0 && lane == 0) {
      const uint32_t smem0 = smem_u32(smem);
      const uint64_t desc0 = smem_desc_sw128(smem0);
      const uint32_t idesc = idesc_mxf4_pair(ncols);
      const uint32_t sf = tmem_base + kFp4SfCol;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t g = 0;  // one per (tile, segment), as on the producer side
      const int nseg = kSeg ? prm.nseg : 1;
      constexpr int G = (8 << LG) / 256;  // k-blocks per macro step
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters) {
        const TileCoord tc = tile_coord<kSplit>(prm, tile);
        const int64_t nkb_seg = kSeg ? prm.nkb_seg : (int64_t)(tc.mc1 - tc.mc0) * G;
        for (int seg = 0; seg < nseg && ok; ++seg, ++g) {
          if (g > 0) ok = mbar_wait_cl(b.tempty, (uint32_t)((g - 1) & 1), b.abort);
          if (!ok) break;
          tc_fence_after();
          for (int64_t kb = 0; kb < nkb_seg; ++kb) {
            if (!mbar_wait(&b.full[stage], phase, b.abort) ||
                !mbar_wait_cl(&b.pfull[stage], phase, b.abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t dst = desc_add(desc0, (uint32_t)stage * Cfg::kStage);
            const uint32_t acc0 = kb > 0 ? 1u : 0u;
#pragma unroll
            for (int kk = 0; kk < kKB / 32; ++kk) {  // 32 bytes = 64 positions per MMA
              if (kk >= prm.mma_ksteps) break;  // past every window of the launch
              const uint64_t bdesc = desc_add(dst, Cfg::kStageA + kk * 32);
#pragma unroll
              for (int j = 0; j < kAcc; ++j) {
                const uint64_t adesc = desc_add(dst, j * (128 * kKB) + kk * 32);
                // a and b read their (all-equal) scale factors from the same columns
                tc_mma_mxf4_pair(tmem_base + (uint32_t)(j * ncols), adesc, bdesc, idesc, sf, sf,
                                 kk > 0 ? 1u : acc0);
              }
            }
            tc_commit_pair_both(&b.empty[stage]);
            if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          tc_commit_pair_both(b.tfull);
        }
      }
      tc_commit_pair_local(b.drain);
      mbar_wait_own_cl(b.drain, 0);
    } else if (rank == 1 && lane == 0) {
      // ============ forwarder (odd CTA): each filled stage of this CTA is
      // announced to the MMA thread with one cluster-scope release
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      constexpr int G = (8 << LG) / 256;
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters) {
        const TileCoord tc = tile_coord<kSplit>(prm, tile);
        const int64_t nkb = (int64_t)(tc.mc1 - tc.mc0) * G;
        for (int64_t kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&b.full[stage], phase, b.abort)) { ok = false; break; }
          mbar_arrive_cluster(b.pfull_cl + 8u * (uint32_t)stage);
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (kPackedB && warp == kTmaWarp) {
    // ========================== b loader (lane 0): prepacked rows by TMA
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      const uint32_t smem0 = smem_u32(smem);
      const uint32_t bytes = (uint32_t)(ncols / 2) * kKB;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t it = 0;
      constexpr int G = (8 << LG) / 256;
      for (int64_t tile = cluster; tile < prm.tiles && ok; tile += nclusters, ++it) {
        const TileCoord tc = tile_coord<kSplit>(prm, tile);
        const int64_t rem = tc.rem;
        const int kb0 = tc.mc0 * G;
        const int64_t nkb = (int64_t)(tc.mc1 - tc.mc0) * G;
        const int nb0 = (int)((rem / prm.tiles_m) * ncols + (int64_t)rank * (ncols / 2));
        // the previous tile's epilogue stages its transpose in the ring (the
        // epi barrier completes once per segment: the epilogue is the tile's
        // last completion)
        const int64_t epi_done = it * (kSeg ? prm.nseg : 1) - 1;
        if (it > 0 && !mbar_wait(b.epi, (uint32_t)(epi_done & 1), b.abort)) break;
        for (int64_t kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&b.empty[stage], phase ^ 1, b.abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&b.full[stage], bytes);
          tma_load_2d(smem0 + stage * Cfg::kStage + Cfg::kStageA, &tmap,
                      (int)((kb0 + kb) * kKB), nb0, &b.full[stage]);
          // (qkv_proj shape: 2.9 % faster than without; 8 k-blocks ahead: 2.6 %)
          if (kb + kL2Ahead < nkb)
            tma_prefetch_l2_2d(&tmap, (int)((kb0 + kb + kL2Ahead) * kKB), nb0);
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else {
    // ============================ producers + epilogue (kProducerWarps warps)
    const uint32_t smem_s = smem_u32(smem);
    ProdState st{0, 0u, 0};
    int64_t it = 0;
    const int half = ncols / 2;
    for (int64_t tile = cluster; tile < prm.tiles; tile += nclusters, ++it) {
      const TileCoord tc = tile_coord<kSplit>(prm, tile);
      const int64_t slice = tc.slice;
      const int64_t rem = tc.rem;
      constexpr int64_t kRowsA = kOneAcc ? 128 : 256;  // a rows per CTA
      const int64_t m0 = (rem % prm.tiles_m) * (2 * kRowsA) + (int64_t)rank * kRowsA;
      const int64_t n0 = (rem / prm.tiles_m) * ncols;
      const int64_t slice_b = prm.P.batch_b == 1 ? 0 : slice;
      if (!produce_rows_fp4<LG, Cfg::kStages, kPackedB, kOneAcc, false, kSeg>(
              prm, b, st, smem_s, Cfg::kStageA, lane, slice, slice_b, m0,
              n0 + (int64_t)rank * half, half, tmem_base, warp, n0, kSplit ? tc.mc0 : 0,
              kSplit ? tc.mc1 : -1))
        break;
      int32_t *part = kSplit ? prm.part + tc.split * prm.part_stride : nullptr;
      if (!tile_epilogue<256, kSeg, true, true, kOneAcc>(prm, b, st, smem, tmem_base, warp, lane,
                                                         slice, slice_b, m0, n0, it, part))
        break;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while the pair may still touch its memory
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
  }
  if (threadIdx.x == 0 && *b.abort) atomicOr(prm.error, 1u);
}

// ---------------------------------------------------------------------------
// Narrow e2m1 tiles on one CTA (N <= 128, e.g. Attn@V per head): 256 a rows as
// two M = 128 accumulators x BN columns (fp32) in TMEM columns [0, 2 BN), the
// unit scale factors at kFp4SfCol, kind::mxf4 MMAs of cta_group::1.  With the
// b side this narrow a CTA pair would only split its few b rows, while each
// stage's fixed costs (barriers, the cross-CTA hop) would be paid on half the
// a rows; here a stage carries 256 a rows x 256 positions.
template <int BN>
struct Fp4NarrowCfg {
  static constexpr uint32_t kStageA = kBM * kKB;  // 32 KB
  static constexpr uint32_t kStage = kStageA + BN * kKB;
  static constexpr int kStages = 4;
  static constexpr size_t kSmem = (size_t)kStages * kStage + 1024 /*align*/ + 256;
  static_assert(kStages * kStage >= kEpiStagingBytes, "the ring holds the epilogue staging");
  static_assert(2 * BN <= (int)kFp4SfCol, "accumulators below the scale factors");
};

__host__ __device__ constexpr uint32_t idesc_mxf4_m128(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
         ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void tc_mma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t tmem_sf, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%5], "
      "p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tmem_sf)
      : "memory");
}

template <int BN, int LG>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_fp4_narrow_kernel(const TcParams prm) {
  using Cfg = Fp4NarrowCfg<BN>;
  constexpr uint32_t kTmemAlloc = 512;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars b;
  b.full = reinterpret_cast<uint64_t *>(smem + Cfg::kStages * Cfg::kStage);
  b.empty = b.full + Cfg::kStages;
  b.tfull = b.empty + Cfg::kStages;
  b.tempty = b.tfull + 1;
  b.drain = b.tempty + 1;
  b.epi = b.drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(b.epi + 1);
  b.abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&b.full[s], kProducerWarps);
      mbar_init(&b.empty[s], 1);
    }
    mbar_init(b.tfull, 1);
    mbar_init(b.tempty, kProducers);
    mbar_init(b.drain, 1);
    mbar_init(b.epi, kProducers);
    *b.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // unit scale factors in columns [kFp4SfCol, 512) of every lane
  if (warp >= 1 && warp <= 4) {
    uint32_t one[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) one[i] = 0x7F7F7F7Fu;
    const uint32_t t = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + kFp4SfCol;
    tmem_st16(t, one);
    tmem_st16(t + 16, one);
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    // ================================================= MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_mxf4_m128(BN);
      const uint32_t smem0 = smem_u32(smem);
      const uint64_t desc0 = smem_desc_sw128(smem0);
      const uint32_t sf = tmem_base + kFp4SfCol;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t g = 0;
      for (int64_t tile = blockIdx.x; tile < prm.tiles && ok; tile += gridDim.x, ++g) {
        if (g > 0) ok = mbar_wait(b.tempty, (uint32_t)((g - 1) & 1), b.abort);
        if (!ok) break;
        tc_fence_after();
        for (int64_t kb = 0; kb < prm.nkb; ++kb) {
          if (!mbar_wait(&b.full[stage], phase, b.abort)) { ok = false; break; }
          tc_fence_after();
          const uint64_t dst = desc_add(desc0, (uint32_t)stage * Cfg::kStage);
          const uint32_t acc0 = kb > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < kKB / 32; ++kk) {  // 32 bytes = 64 positions per MMA
            if (kk >= prm.mma_ksteps) break;  // past every window of the launch
            const uint64_t bdesc = desc_add(dst, Cfg::kStageA + kk * 32);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint64_t adesc = desc_add(dst, j * (128 * kKB) + kk * 32);
              tc_mma_mxf4(tmem_base + (uint32_t)(j * BN), adesc, bdesc, idesc, sf,
                          kk > 0 ? 1u : acc0);
            }
          }
          tc_commit(&b.empty[stage]);
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(b.tfull);
      }
      tc_commit(b.drain);
      mbar_wait_own(b.drain, 0);
    }
    __syncwarp();
  } else {
    // ============================ producers + epilogue (kProducerWarps warps)
    const uint32_t smem_s = smem_u32(smem);
    ProdState st{0, 0u, 0};
    int64_t it = 0;
    for (int64_t tile = blockIdx.x; tile < prm.tiles; tile += gridDim.x, ++it) {
      const int64_t slice = tile / (prm.tiles_m * prm.tiles_n);
      const int64_t rem = tile % (prm.tiles_m * prm.tiles_n);
      const int64_t m0 = (rem % prm.tiles_m) * kBM;
      const int64_t n0 = (rem / prm.tiles_m) * BN;
      const int64_t slice_b = prm.P.batch_b == 1 ? 0 : slice;
      if (!produce_rows_fp4<LG, Cfg::kStages, false, false, true>(
              prm, b, st, smem_s, Cfg::kStageA, lane, slice, slice_b, m0, n0, BN))
        break;
      if (!tile_epilogue<BN, false, false, true>(prm, b, st, smem, tmem_base, warp, lane, slice,
                                                 slice_b, m0, n0, it))
        break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
  }
  if (threadIdx.x == 0 && *b.abort) atomicOr(prm.error, 1u);
}

// ---------------------------------------------------------------------------
// Sum of the K splits' exact int32 partial counts, rescaled as the tile
// epilogue would (per-row factor, row and column scales, bias, output type).
__global__ void split_reduce_kernel(const GemmProblem P, const int32_t *__restrict__ part,
                                    int ksplit, int64_t stride, int64_t m_rows, int64_t n_rows) {
  const int64_t per_slice = m_rows * n_rows;
  const int64_t total = P.batch * per_slice;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slice = i / per_slice, r = i % per_slice;
    const int64_t m = r / n_rows, n = r % n_rows;
    const int64_t grow = slice * P.M + m;
    const int L = row_stream_len(P, slice, grow);
    if (L < 0) continue;  // the row belongs to another call
    const int64_t o = grow * P.N + n;
    int32_t acc = 0;
    for (int sp = 0; sp < ksplit; ++sp) acc += part[sp * stride + o];
    float y = 0.0f;
    if (L > 0) {
      const int64_t rb = (P.batch_b == 1 ? 0 : slice) * P.N + n;
      y = sc_rescale_f(P.mode, sc_rescale_factor(P.mode, P.prec, L), acc, P.K, P.qa.scale[grow],
                       P.qa.zero[grow], P.qa.rowsum[grow], P.qb.scale[rb], P.qb.zero[rb],
                       P.qb.rowsum[rb]);
    } else {
      acc = 0;
    }
    if (P.bias) y = __fadd_rn(y, P.bias[n]);
    store_out(P, o, y);
    if (P.acc_out) P.acc_out[o] = acc;
  }
}

// ---------------------------------------------------------------------------
// Rate probe of the e2m1 MMA the engine's tiles are built from: one CTA per
// SM, one thread issues `iters` x 4 back-to-back kind::mxf4 MMAs of
// M = 128 x N = BN x K = 64 (unit block scales, zero operands in shared
// memory) into one TMEM accumulator, then waits for them with a bounded wait.
// Nothing else runs, so the launch time is the MMA pipe's time.
template <int BN>
__global__ void __launch_bounds__(128, 1) probe_mma_mxf4_kernel(int iters, unsigned int *error) {
  constexpr uint32_t kA = 128 * kKB, kB = BN * kKB;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *done = reinterpret_cast<uint64_t *>(smem + kA + kB);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  const int warp = threadIdx.x >> 5;
  for (uint32_t i = threadIdx.x; i < (kA + kB) / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_async_smem();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  {  // unit scale factors in columns [kFp4SfCol, 512), warp w covers lanes 32 w ..
    uint32_t one[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) one[i] = 0x7F7F7F7Fu;
    const uint32_t t = tmem_base + ((uint32_t)(warp * 32) << 16) + kFp4SfCol;
    tmem_st16(t, one);
    tmem_st16(t + 16, one);
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(smem), b0 = a0 + kA;
    constexpr uint32_t idesc = idesc_mxf4_m128(BN);
    const uint32_t sf = tmem_base + kFp4SfCol;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < kKB / 32; ++kk)
        tc_mma_mxf4(tmem_base, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), idesc,
                    sf, (it > 0 || kk > 0) ? 1u : 0u);
    }
    tc_commit(done);
    // the issued MMAs always complete: wait for them before the TMEM is freed
    mbar_wait_own(done, 0);
    if (!mbar_try_wait(done, 0)) atomicOr(error, 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(512u));
  }
}

template <int BN, int kProd, int LG, bool kSeg>
cudaError_t launch_bn(TcParams prm, int sms, cudaStream_t s) {
  const size_t smem = TcCfg<BN>::smem_bytes(kProd == kProdTable);
  auto kern = gemm_tc_kernel<BN, kProd, LG, kSeg>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  prm.rep = 0x01010101u;
  prm.stage_bytes = TcCfg<BN>::kStage;
  const int64_t grid = prm.tiles < sms ? prm.tiles : sms;
  kern<<<(unsigned)grid, kThreads, smem, s>>>(prm);
  return cudaGetLastError();
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <int LG, bool kPackedB>
cudaError_t launch_pair_v(TcParams prm, int dev, const CUtensorMap &tmap, cudaStream_t s) {
  auto kern = gemm_tc_pair_kernel<LG, kPackedB>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads + (kPackedB ? 32 : 0), 1, 1);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // one cluster per resident pair slot (persistent tiles)
  static int max_clusters[64] = {};
  int clusters = dev >= 0 && dev < 64 ? max_clusters[dev] : 0;
  if (clusters <= 0) {
    cfg.gridDim = dim3(2, 1, 1);
    if ((e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg)) != cudaSuccess) return e;
    if (clusters <= 0) return cudaErrorInvalidConfiguration;
    if (dev >= 0 && dev < 64) max_clusters[dev] = clusters;
  }
  const int64_t grid = prm.tiles < clusters ? prm.tiles : clusters;
  cfg.gridDim = dim3((unsigned)(2 * grid), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, prm, tmap);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int LG>
cudaError_t launch_pair(TcParams prm, int dev, cudaStream_t s) {
  prm.rep = 0x01010101u;
  prm.stage_bytes = kPairStage;
  // pair tiles: 512 a rows x 256 b rows
  prm.tiles_m = (prm.m_rows + 2 * kBM - 1) / (2 * kBM);
  prm.tiles_n = (prm.n_rows + 255) / 256;
  prm.tiles = prm.P.batch * prm.tiles_m * prm.tiles_n;
  CUtensorMap tmap;
  memset(&tmap, 0, sizeof(tmap));
  // prepacked b (bytes laid out at Lp = 2^prec) serves calls whose padded
  // stream length is the full 2^prec
  const GemmProblem &P = prm.P;
  if (P.b_streams && !P.b_e2m1 && P.batch_b == 1 && LG == P.prec) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc) {
      const cuuint64_t row_bytes = (cuuint64_t)(P.ldk << LG);
      cuuint64_t gdim[2] = {row_bytes, (cuuint64_t)P.N};
      cuuint64_t gstride[1] = {row_bytes};
      cuuint32_t box[2] = {(cuuint32_t)kKB, 128u};
      cuuint32_t estride[2] = {1u, 1u};
      const CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                             const_cast<uint8_t *>(P.b_streams), gdim, gstride, box, estride,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r == CUDA_SUCCESS) return launch_pair_v<LG, true>(prm, dev, tmap, s);
    }
    // no encoder or a rejected map: generate b from the packed codes instead
  }
  return launch_pair_v<LG, false>(prm, dev, tmap, s);
}

// b rows per e2m1 pair tile: fewest computed columns with a per-tile cost of
// 32 columns (epilogue, a rows generated again), the wider tile on ties.  One
// accumulator leaves room for 256 columns; a b side that fits one tile is
// taken whole (a multiple of 16, at least 16: the M = 256 MMA's N).
// Segmented tiles keep fp32 running sums next to the accumulator, so they
// also stay within kFp4MaxCols.
int fp4_tile_cols(int64_t n_rows, bool one_acc, bool seg = false) {
  const int max_cols = one_acc && !seg ? 256 : kFp4MaxCols;
  if (n_rows <= max_cols) return n_rows <= 16 ? 16 : (int)((n_rows + 15) / 16 * 16);
  int best = max_cols;
  int64_t best_cost = -1;
  for (int nt = max_cols; nt >= 128; nt -= 16) {
    const int64_t cost = ((n_rows + nt - 1) / nt) * (nt + 32);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = nt;
    }
  }
  return best;
}

template <int LG, bool kPackedB, bool kOneAcc, bool kSeg = false, bool kSplit = false>
cudaError_t launch_pair_fp4_v(const TcParams &prm, int dev, const CUtensorMap &tmap,
                              cudaStream_t s) {
  auto kern = gemm_tc_pair_fp4_kernel<LG, kPackedB, kOneAcc, kSeg, kSplit>;
  constexpr size_t kSmem = Fp4PairCfg<kOneAcc, kSeg ? kSegPairStages : kPairStages>::kSmem;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads + (kPackedB ? 32 : 0), 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_clusters[64] = {};
  int clusters = dev >= 0 && dev < 64 ? max_clusters[dev] : 0;
  if (clusters <= 0) {
    cfg.gridDim = dim3(2, 1, 1);
    if ((e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg)) != cudaSuccess) return e;
    if (clusters <= 0) return cudaErrorInvalidConfiguration;
    if (dev >= 0 && dev < 64) max_clusters[dev] = clusters;
  }
  const int64_t grid = prm.tiles < clusters ? prm.tiles : clusters;
  cfg.gridDim = dim3((unsigned)(2 * grid), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, prm, tmap);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int LG, bool kOneAcc>
cudaError_t launch_pair_fp4(TcParams prm, int dev, cudaStream_t s, int ksplit) {
  prm.rep = 0x01010101u;
  prm.stage_bytes = Fp4PairCfg<kOneAcc>::kStage;
  prm.ncols = fp4_tile_cols(prm.n_rows, kOneAcc);
  prm.nkb = (prm.P.ldk << LG) / 256;  // 256 stream positions per stage
  prm.nkb_seg = prm.nkb;
  const int64_t rows_tile = kOneAcc ? 256 : 2 * kBM;
  prm.tiles_m = (prm.m_rows + rows_tile - 1) / rows_tile;
  prm.tiles_n = (prm.n_rows + prm.ncols - 1) / prm.ncols;
  prm.tiles = prm.P.batch * prm.tiles_m * prm.tiles_n;
  if (ksplit > 1) {
    const int nmacro = (int)(prm.P.ldk >> 3);
    prm.msplit = (nmacro + ksplit - 1) / ksplit;
    prm.ksplit = (nmacro + prm.msplit - 1) / prm.msplit;
    prm.tiles_split = prm.tiles;
    prm.tiles *= prm.ksplit;
    prm.part = prm.P.split_part;
    prm.part_stride = prm.P.batch * prm.P.M * prm.P.N;
  }
  CUtensorMap tmap;
  memset(&tmap, 0, sizeof(tmap));
  // prepacked e2m1 b (positions laid out at Lp = 2^prec) serves calls whose
  // padded stream length is the full 2^prec
  const GemmProblem &P = prm.P;
  if (P.b_streams && P.b_e2m1 && P.batch_b == 1 && LG == P.prec) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc) {
      const cuuint64_t row_bytes = (cuuint64_t)((P.ldk << LG) / 2);
      cuuint64_t gdim[2] = {row_bytes, (cuuint64_t)P.N};
      cuuint64_t gstride[1] = {row_bytes};
      cuuint32_t box[2] = {(cuuint32_t)kKB, (cuuint32_t)(prm.ncols / 2)};
      cuuint32_t estride[2] = {1u, 1u};
      const CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                             const_cast<uint8_t *>(P.b_streams), gdim, gstride, box, estride,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r == CUDA_SUCCESS)
        return prm.ksplit > 1 ? launch_pair_fp4_v<LG, true, kOneAcc, false, true>(prm, dev, tmap, s)
                              : launch_pair_fp4_v<LG, true, kOneAcc>(prm, dev, tmap, s);
    }
    // no encoder or a rejected map: generate b from the packed codes instead
  }
  return prm.ksplit > 1 ? launch_pair_fp4_v<LG, false, kOneAcc, false, true>(prm, dev, tmap, s)
                        : launch_pair_fp4_v<LG, false, kOneAcc>(prm, dev, tmap, s);
}

// Segmented K on the e2m1 pairs (head-aligned compensation, chunk-D): one
// accumulator per CTA, a segment = kseg * Lp / 256 whole stages; b by TMA from
// a prepacked segmented weight at Lp = 2^prec, else generated from its
// per-segment codes.
template <int LG>
cudaError_t launch_pair_fp4_seg(TcParams prm, int dev, cudaStream_t s) {
  prm.rep = 0x01010101u;
  prm.stage_bytes = Fp4PairCfg<true, kSegPairStages>::kStage;
  prm.ncols = fp4_tile_cols(prm.n_rows, true, true);
  prm.nkb = (prm.P.ldk << LG) / 256;
  prm.nkb_seg = (prm.P.kseg << LG) / 256;
  prm.tiles_m = (prm.m_rows + 255) / 256;
  prm.tiles_n = (prm.n_rows + prm.ncols - 1) / prm.ncols;
  prm.tiles = prm.P.batch * prm.tiles_m * prm.tiles_n;
  CUtensorMap tmap;
  memset(&tmap, 0, sizeof(tmap));
  const GemmProblem &P = prm.P;
  if (P.b_streams && P.b_e2m1 && P.batch_b == 1 && LG == P.prec) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc) {
      const cuuint64_t row_bytes = (cuuint64_t)((P.ldk << LG) / 2);
      cuuint64_t gdim[2] = {row_bytes, (cuuint64_t)P.N};
      cuuint64_t gstride[1] = {row_bytes};
      cuuint32_t box[2] = {(cuuint32_t)kKB, (cuuint32_t)(prm.ncols / 2)};
      cuuint32_t estride[2] = {1u, 1u};
      const CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                             const_cast<uint8_t *>(P.b_streams), gdim, gstride, box, estride,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r == CUDA_SUCCESS) return launch_pair_fp4_v<LG, true, true, true>(prm, dev, tmap, s);
    }
  }
  return launch_pair_fp4_v<LG, false, true, true>(prm, dev, tmap, s);
}

template <int BN, int LG>
cudaError_t launch_fp4_narrow_lg(TcParams prm, int sms, cudaStream_t s) {
  using Cfg = Fp4NarrowCfg<BN>;
  auto kern = gemm_tc_fp4_narrow_kernel<BN, LG>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
  if (e != cudaSuccess) return e;
  prm.rep = 0x01010101u;
  prm.stage_bytes = Cfg::kStage;
  prm.ncols = BN;
  prm.nkb = (prm.P.ldk << LG) / 256;  // 256 stream positions per stage
  prm.nkb_seg = prm.nkb;
  const int64_t grid = prm.tiles < sms ? prm.tiles : sms;
  kern<<<(unsigned)grid, kThreads, Cfg::kSmem, s>>>(prm);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_fp4_narrow(const TcParams &prm, int sms, cudaStream_t s) {
  if (prm.lp_log2 == 7) return launch_fp4_narrow_lg<BN, 7>(prm, sms, s);
  return launch_fp4_narrow_lg<BN, 8>(prm, sms, s);
}

template <int BN, int LG>
cudaError_t launch_ts_lg(TcParams prm, int sms, cudaStream_t s) {
  const size_t smem = TsCfg<BN>::smem_bytes;
  auto kern = gemm_tc_ts_kernel<BN, LG>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  prm.rep = 0x01010101u;
  prm.stage_bytes = TsCfg<BN>::kStageB;
  const int64_t grid = prm.tiles < sms ? prm.tiles : sms;
  kern<<<(unsigned)grid, kThreads, smem, s>>>(prm);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_ts(const TcParams &prm, int sms, cudaStream_t s) {
  if (prm.lp_log2 == 6) return launch_ts_lg<BN, 6>(prm, sms, s);
  if (prm.lp_log2 == 7) return launch_ts_lg<BN, 7>(prm, sms, s);
  return launch_ts_lg<BN, 8>(prm, sms, s);
}

template <int BN, bool kSeg>
cudaError_t launch_rows(const TcParams &prm, int sms, cudaStream_t s) {
  if (prm.lp_log2 == 6) return launch_bn<BN, kProdRows, 6, kSeg>(prm, sms, s);
  if (prm.lp_log2 == 7) return launch_bn<BN, kProdRows, 7, kSeg>(prm, sms, s);
  return launch_bn<BN, kProdRows, 8, kSeg>(prm, sms, s);
}

// Enable-window rows for the table path: [sign 0/1][window 0..128] x 128
// bytes, byte t = (t < window) ? (sign ? -1 : +1) : 0.  Copied into shared
// memory by every CTA; a producer copies chunk c of row (sign, window).
constexpr size_t kThermBytes = (size_t)2 * 129 * 128;
__device__ __align__(128) unsigned char g_therm[kThermBytes];
std::mutex g_therm_mu;
SymbolCache g_therm_ptr[kMaxCachedDevices];

// Filled on first use per (device, context); the cache key follows
// cached_symbol_address.
const unsigned char *therm_table(cudaError_t *err) {
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess || dev < 0 || dev >= kMaxCachedDevices) return nullptr;
  void *ctx = current_context();
  std::lock_guard<std::mutex> lock(g_therm_mu);
  SymbolCache &c = g_therm_ptr[dev];
  if (!c.ptr || c.ctx != ctx) {
    std::vector<unsigned char> h(kThermBytes, 0);
    for (int sg = 0; sg < 2; ++sg)
      for (int q = 0; q <= 128; ++q) {
        unsigned char *row = h.data() + ((size_t)(sg * 129 + q) << 7);
        for (int t = 0; t < 128; ++t) row[t] = t < q ? (sg ? 0xFF : 0x01) : 0x00;
      }
    if ((*err = cudaMemcpyToSymbol(g_therm, h.data(), kThermBytes)) != cudaSuccess) return nullptr;
    void *p = nullptr;
    if ((*err = cudaGetSymbolAddress(&p, g_therm)) != cudaSuccess) return nullptr;
    c.ptr = p;
    c.ctx = ctx;
  }
  return static_cast<const unsigned char *>(c.ptr);
}

}  // namespace

namespace {
int padded_stream_log2(const GemmProblem &P) {
  const int T = 1 << P.prec;
  const int Lmax = (P.row_L || P.slice_L) ? T : P.stoc_len;
  int lg = 5;
  while ((1 << lg) < Lmax) ++lg;
  return lg;
}
}  // namespace

bool tc_supported(const GemmProblem &P) {
  if (P.prec < 5 || P.prec > 8) return false;           // pool rows >= 32 bytes
  if (P.ldk * 256 >= (int64_t)1 << 31) return false;    // 32-bit k-block index math
  if (P.mode == SCMP_UNIPOLAR && P.prec == 8) return false;  // 8-bit thresholds
  if (P.nseg == 1) return P.pool_dims >= P.K;           // reduction index = pool row
  // segmented K: whole k-blocks per segment, pool row = index inside segment;
  // the per-segment counts are not summed into acc_out on this engine
  if (P.pool_dims < P.kseg || P.acc_out) return false;
  return ((P.kseg << padded_stream_log2(P)) % kKB) == 0;
}

int tc_stream_log2(const GemmProblem &P) { return padded_stream_log2(P); }

bool tc_row_producers(const GemmProblem &P) {
  const int lg = padded_stream_log2(P);
  if (lg < 6 || lg > 8 || (P.ldk & 7) != 0) return false;
  if (P.nseg > 1 && (P.kseg & 7) != 0) return false;  // segments end on macro steps
  // 16-byte code loads: rows of ldk int16 codes from 16-byte aligned planes
  // (pool complement rows cover the padded indices)
  return ((reinterpret_cast<uintptr_t>(P.qa.code) | reinterpret_cast<uintptr_t>(P.qb.code)) & 15) ==
         0;
}

int tc_block_n(int64_t N) { return N <= 64 ? 64 : (N <= 128 ? 128 : 256); }

// The e2m1 CTA pairs take every row-producer problem with one K segment at
// Lp = 128 / 256 whose counts stay below 2^24 (exact in fp32), unless b comes
// prepacked as int8 bytes (prepacked e2m1 bytes are loaded by TMA when
// Lp = 2^prec, else b is generated from the packed codes).
bool tc_nibble_pairs(const GemmProblem &P, int64_t m_rows, int64_t n_rows) {
  (void)m_rows;
  (void)n_rows;
  const int lg = padded_stream_log2(P);
  if (!tc_row_producers(P) || (lg != 7 && lg != 8)) return false;
  if (P.nseg > 1)  // segments of whole 256-position stages
    return (P.b_streams == nullptr || P.b_e2m1) && ((P.kseg << lg) % 256) == 0 &&
           (P.kseg << lg) < (1LL << 24);
  return (P.b_streams == nullptr || P.b_e2m1) && (P.ldk << lg) < (1LL << 24);
}

int tc_ksplit(const GemmProblem &P, int64_t m_rows, int64_t n_rows) {
  if (m_rows <= 0 || n_rows <= 128 || P.nseg != 1 || P.batch <= 0) return 1;
  if (!tc_supported(P) || !tc_nibble_pairs(P, m_rows, n_rows)) return 1;
  const bool two = m_rows > kBM;
  const int ncols = fp4_tile_cols(n_rows, !two);
  const int64_t rows_tile = two ? 2 * kBM : kBM;
  const int64_t tiles =
      P.batch * ((m_rows + rows_tile - 1) / rows_tile) * ((n_rows + ncols - 1) / ncols);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t pairs = sms / 2;
  if (2 * tiles > pairs) return 1;  // the output tiles already fill half of the pairs
  const int64_t nmacro = P.ldk >> 3;
  int64_t ks = pairs / tiles;
  if (ks > nmacro / 4) ks = nmacro / 4;  // at least 32 reduction indices per split
  if (ks < 2) return 1;
  const int64_t msplit = (nmacro + ks - 1) / ks;
  return (int)((nmacro + msplit - 1) / msplit);
}

int tc_tile_n(const GemmProblem &P, int64_t N) {
  const int bn = tc_block_n(N);
  return (P.nseg > 1 && bn > 128) ? 128 : bn;
}

cudaError_t launch_gemm_tc(const GemmProblem &P, int64_t m_rows, int64_t n_rows,
                           unsigned int *error, cudaStream_t s, int *launches) {
  *launches = 0;
  if (P.M == 0 || P.N == 0 || P.batch == 0 || m_rows == 0 || n_rows == 0) return cudaSuccess;
  *launches = 1;
  TcParams prm{};
  prm.P = P;
  const int lg = padded_stream_log2(P);
  prm.lp_log2 = lg;
  prm.shift_pool = (P.mode == SCMP_BIPOLAR && P.prec == 8) ? 1 : 0;
  // row producers run every padded index (ldk); chunk producers stop at K
  const int64_t krun = tc_row_producers(P) ? P.ldk : P.K;
  prm.nkb = (krun * ((int64_t)1 << lg) + kKB - 1) / kKB;
  prm.nseg = P.nseg;
  prm.kseg = (int)P.kseg;
  prm.nkb_seg = P.nseg > 1 ? ((P.kseg << lg) / kKB) : prm.nkb;
  prm.m_rows = m_rows;
  prm.n_rows = n_rows;
  prm.mma_ksteps = 4;
  if (lg == 8 && !P.row_L && !P.slice_L) {
    // the longest window of the launch: |code| <= 2^p - 1 at L = stoc_len
    const int64_t kmax = ((((int64_t)1 << P.prec) - 1) * P.stoc_len) >> P.prec;
    const int steps = (int)((kmax + 63) / 64);
    prm.mma_ksteps = steps < 1 ? 1 : (steps > 4 ? 4 : steps);
  }
  const int bn = tc_tile_n(P, n_rows);
  prm.tiles_m = (m_rows + kBM - 1) / kBM;
  prm.tiles_n = (n_rows + bn - 1) / bn;
  prm.tiles = P.batch * prm.tiles_m * prm.tiles_n;
  prm.error = error;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (tc_row_producers(P)) {
    // pairs pay off only with two a tiles per pair (one accumulator per CTA
    // would generate as many rows per MAC as a single CTA)
    if (tc_nibble_pairs(P, m_rows, n_rows)) {
      if (P.nseg > 1) {
        // one accumulator per CTA (256 x <= 240 tiles): two accumulators leave
        // room for 112 columns only, and measured slower on the compensation
        if (lg == 7) return launch_pair_fp4_seg<7>(prm, dev, s);
        return launch_pair_fp4_seg<8>(prm, dev, s);
      }
      // narrow b on one CTA (prepacked int8-free b is generated from codes)
      if (n_rows <= 128) {
        if (bn == 64) return launch_fp4_narrow<64>(prm, sms, s);
        return launch_fp4_narrow<128>(prm, sms, s);
      }
      // two accumulators (512-row tiles) when both sides are wide; K splits
      // (with their reduce) when the tiles would leave most pairs idle
      const bool two = m_rows > kBM && n_rows > 128;
      const int ks = P.split_part ? tc_ksplit(P, m_rows, n_rows) : 1;
      cudaError_t e;
      if (lg == 7)
        e = two ? launch_pair_fp4<7, false>(prm, dev, s, ks) : launch_pair_fp4<7, true>(prm, dev, s, ks);
      else
        e = two ? launch_pair_fp4<8, false>(prm, dev, s, ks) : launch_pair_fp4<8, true>(prm, dev, s, ks);
      if (e != cudaSuccess || ks <= 1) return e;
      const int64_t total = P.batch * m_rows * n_rows;
      int64_t blocks = (total + 255) / 256;
      if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
      split_reduce_kernel<<<(unsigned)blocks, 256, 0, s>>>(P, P.split_part, ks,
                                                           P.batch * P.M * P.N, m_rows, n_rows);
      *launches = 2;
      return cudaGetLastError();
    }
    if (P.nseg == 1 && bn == 256 && m_rows > kBM) {
      if (lg == 6) return launch_pair<6>(prm, dev, s);
      if (lg == 7) return launch_pair<7>(prm, dev, s);
      return launch_pair<8>(prm, dev, s);
    }
    if (P.nseg > 1) {
      if (bn == 64) return launch_rows<64, true>(prm, sms, s);
      return launch_rows<128, true>(prm, sms, s);
    }
    // narrow tiles: the window operand goes through TMEM, not shared memory
    if (bn == 64) return launch_ts<64>(prm, sms, s);
    if (bn == 128) return launch_ts<128>(prm, sms, s);
    return launch_rows<256, false>(prm, sms, s);
  }
  if (P.nseg > 1) {
    if (bn == 64) return launch_bn<64, kProdChunks, 0, true>(prm, sms, s);
    return launch_bn<128, kProdChunks, 0, true>(prm, sms, s);
  }
  // Table path: every k-block lies inside one reduction index, and the tile is
  // narrow, so enable windows dominate the operand generation.
  if (lg >= 7 && bn == 64) {
    cudaError_t e;
    prm.therm = therm_table(&e);
    if (!prm.therm) return e != cudaSuccess ? e : cudaErrorUnknown;
    return launch_bn<64, kProdTable, 0, false>(prm, sms, s);
  }
  if (bn == 64) return launch_bn<64, kProdChunks, 0, false>(prm, sms, s);
  if (bn == 128) return launch_bn<128, kProdChunks, 0, false>(prm, sms, s);
  return launch_bn<256, kProdChunks, 0, false>(prm, sms, s);
}

namespace {
template <typename T>
int set_device_word(const T &symbol, const T &value, const char *what) {
  const cudaError_t e = cudaMemcpyToSymbol(symbol, &value, sizeof(T));
  if (e != cudaSuccess) {
    char buf[200];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    set_last_error(buf);
    return SCMP_ECUDA;
  }
  return SCMP_OK;
}
}  // namespace

int debug_set_wait_limit(uint64_t ns) {
  if (ns == 0) {
    set_last_error("the wait limit must be positive");
    return SCMP_EINVAL;
  }
  const unsigned long long v = ns;
  return set_device_word(g_wait_limit_ns, v, "setting the wait limit");
}

cudaError_t launch_probe_mma_mxf4(int n, int iters, int blocks, unsigned int *error,
                                  cudaStream_t s) {
  // more shared memory than two CTAs can share: one CTA (one TMEM owner) per SM
  const size_t smem = 120 * 1024;
  static_assert((size_t)(128 + 256) * kKB + 1024 + 64 <= 120 * 1024, "probe tiles fit");
  cudaError_t e;
  if (n == 256) {
    if ((e = cudaFuncSetAttribute(probe_mma_mxf4_kernel<256>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
      return e;
    probe_mma_mxf4_kernel<256><<<blocks, 128, smem, s>>>(iters, error);
  } else if (n == 64) {
    if ((e = cudaFuncSetAttribute(probe_mma_mxf4_kernel<64>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
      return e;
    probe_mma_mxf4_kernel<64><<<blocks, 128, smem, s>>>(iters, error);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int debug_hold_producers(int on) {
  const int v = on ? 1 : 0;
  return set_device_word(g_hold_producers, v, "setting the producer hold");
}

}  // namespace scmp
