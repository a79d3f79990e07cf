// fp32-in / fp32-out GEMM on the 5th-generation tensor cores (sm_100a).
//
// The reference multiplies with 32x32 shared-memory tiles, one output per
// thread, and atomics for every `backward` output (bcmm*,
// Engine/kernels.cu:387-539).  This kernel computes the same products with
// tcgen05.mma kind::tf32 as a persistent, warp-specialised kernel (one CTA
// per SM walking the 128 x BN output tiles):
//   * warp 0 (one lane) streams operand tiles through a STAGES-deep shared-
//     memory ring with TMA (cp.async.bulk.tensor, 128-byte swizzle), tracked
//     by mbarriers (full: bytes landed; empty: the MMAs reading the slot
//     retired, signalled by tcgen05.commit);
//   * warp 1 (one lane) issues 128 x BN x 8 MMAs into one of two TMEM
//     accumulators, so a tile's epilogue overlaps the next tile's MMAs;
//   * warps 2-5 drain TMEM with tcgen05.ld, transpose each 32 x 32 block
//     through shared memory and apply the epilogue (assign, += or atomic
//     add, alpha, optional bias) with row-contiguous 128-byte accesses.
// Both K-major and MN-major operands are read straight from their row-major
// storage (instruction-descriptor transpose bits), so dX = dY*W^T and
// dW = X^T*dY need no transposed copies.
//
// Every mbarrier wait is bounded by %globaltimer; on timeout the kernel sets
// the watchdog word, stops issuing work, lets issued copies and MMAs retire,
// frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <cfloat>
#include <type_traits>
#include <stdio.h>
#include <string.h>

#include "gemm.cuh"

namespace mle {

__device__ unsigned int g_tc_watchdog = 0;

namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;                   // fp32 elements per k-block = one 128-byte swizzle row
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA, 4 epilogue warps
constexpr int kEpiLd = 36;                      // staging row pitch (floats): float4-aligned, conflict-free
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s

enum EpiMode { EPI_ASSIGN = 0, EPI_ACCUM = 1, EPI_ATOMIC = 2 };

struct EpiParams {
    float* C;
    const float* bias;
    int64_t ldc;
    int64_t c_stride_b, c_stride_c;  // element offsets per batch / channel index (0 = broadcast)
    int M, N, K;
    int channels;                     // z = (b * channels + c) * splits + split
    int splits, kb_per_split;
    int a_has_b, a_has_c, b_has_b, b_has_c;
    int m_tiles, n_tiles;
    int64_t tiles;                    // m_tiles * n_tiles * batch * channels * splits
    float alpha;
    int mode;
    int vec;                          // C rows (and bias) 16-byte aligned
    int tma_epi;                      // C leaves through bulk tensor stores / reduce-adds (tmC)
    int c_has_b, c_has_c;             // C varies over batch / channel (tensor-map coordinates)
    // implicit convolution (ConvGemm in gemm.cuh); 0 = plain GEMM.
    //   1: k-block kb = (tap, channel block), tap = kb / cv_cblk; B boxes
    //      come from the shifted copies at (p + (kh - pad)*cv_w, c, kw*nb + n)
    //      with p the output pixel (rows of width cv_w, flattened)
    //   2: tile column index = (tap, channel block of BN), tap = n / cv_cblk,
    //      stored as the tile's channel index (C's third coordinate); k = pixel
    //   3: kind 1 with the roles exchanged: tile rows are output pixels
    //      (A = the shifted copies, MN-major), tile columns output channels
    //      (B = the packed weights), C written transposed (c_trans)
    int conv;
    int cv_kw, cv_pad, cv_w, cv_cblk, cv_nb;
    int c_trans;                      // tile rows run along C's contiguous dimension (TMA epilogue only)
    int c_split;                      // > 0: C's inner coordinate is split (x % c_split, x / c_split), 5-D map
    // operand maps of the split view (one copy per operand and stage): a
    // K-major operand as (32 K, rows, K / 32, channel, batch), an MN-major
    // one as (32 MN, K, MN / 32, channel, batch); else the plain 4-D view
    // (MN-major tiles then arrive as one 32-column box each)
    int a_split, b_split;
    // non-null: colsum[n] += sum over this tile's k-range of B[k][n], taken
    // by the epilogue warps from B's stages in shared memory (tiles of the
    // first row-tile only; MN-major B; in a pair each CTA its own columns)
    float* colsum;
};

// Output tile `t` of the persistent walk: n fastest, then m, then (batch,
// channel, split).
struct Tile {
    int m0, n0, bidx, cidx, kb_begin, nkb;
};

// Up to kMaxGroup problems of one layout class share a launch; their tiles
// are numbered consecutively (tile_start is the prefix of ep[g].tiles).
constexpr int kMaxGroup = 3;
struct GemmGroup {
    CUtensorMap a[kMaxGroup], b[kMaxGroup], c[kMaxGroup];
    EpiParams ep[kMaxGroup];
    int64_t tile_start[kMaxGroup + 1];
    int n;
    // kcat > 1: one product over the concatenated reduction of kcat problems
    // that share C, M and N (sum_g A_g B_g); the tiles and the epilogue are
    // problem 0's (ep[0].K = the summed K), k-block kb of a tile reads
    // a[g], b[g] at k-block kb - kcat_kb[g] of segment g
    int kcat;
    int kcat_kb[kMaxGroup + 1];
    // ilv: the problems share their (split, batch, channel, m) tile rows and
    // walk them together, row-tile by row-tile, each problem's n-tiles in
    // turn (ilv_n: prefix of the problems' n_tiles), so tiles that read the
    // same rows of a shared A run back to back and find them in L2
    int ilv;
    int ilv_n[kMaxGroup + 1];
    // some problem sums B's columns: the epilogue warps follow every stage
    // (and release it) as the MMA issuer does
    int colsum;
};

__device__ __forceinline__ int group_of(const GemmGroup& G, int64_t t) {
    int g = 0;
    while (g + 1 < G.n && t >= G.tile_start[g + 1]) ++g;
    return g;
}

// Problem g of tile t and the tile's index within that problem.
__device__ __forceinline__ int locate(const GemmGroup& G, int64_t t, int64_t& tl) {
    if (G.ilv) {
        const int64_t nsum = G.ilv_n[G.n];
        const int64_t outer = t / nsum;
        const int inner = (int)(t - outer * nsum);
        int g = 0;
        while (g + 1 < G.n && inner >= G.ilv_n[g + 1]) ++g;
        tl = outer * (G.ilv_n[g + 1] - G.ilv_n[g]) + (inner - G.ilv_n[g]);
        return g;
    }
    const int g = group_of(G, t);
    tl = t - G.tile_start[g];
    return g;
}

__device__ __forceinline__ Tile tile_at(const EpiParams& ep, int64_t t, int BN, int BMT = 128) {
    Tile x;
    const int n = (int)(t % ep.n_tiles);
    t /= ep.n_tiles;
    const int m = (int)(t % ep.m_tiles);
    int64_t z = t / ep.m_tiles;
    const int split = (int)(z % ep.splits);
    z /= ep.splits;
    x.cidx = (int)(z % ep.channels);
    x.bidx = (int)(z / ep.channels);
    x.m0 = m * BMT;
    x.n0 = n * BN;
    if (ep.conv == 2) {
        x.cidx = n / ep.cv_cblk;
        x.n0 = (n - x.cidx * ep.cv_cblk) * BN;
    }
    const int kb_total = (ep.K + 31) / 32;
    x.kb_begin = split * ep.kb_per_split;
    int kb_end = x.kb_begin + ep.kb_per_split;
    if (kb_end > kb_total) kb_end = kb_total;
    x.nkb = kb_end > x.kb_begin ? kb_end - x.kb_begin : 0;
    return x;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait.  Returns false if the CTA-wide abort flag is (or becomes) set.
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 127u) == 127u) {
            if (*abort_flag) return false;
            const uint64_t now = gtimer();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > kTimeoutNs) {
                *abort_flag = 1;
                atomicOr(&g_tc_watchdog, 1u);
                return false;
            }
        }
    }
}

// Wait that ignores the abort flag (used to drain issued work), still bounded.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > kTimeoutNs) {
            atomicOr(&g_tc_watchdog, 2u);
            return;
        }
    }
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2,
                                            int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

// Epilogue stores: a 32 x 32 fp32 block staged in shared memory (128-byte
// swizzle) leaves with one bulk tensor store, or a bulk tensor reduce-add
// (C += block) for the accumulate and split-K modes.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3,
                                             int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void tma_reduce_add_5d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3, int c4) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.5d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

// One staged 32 x 32 block of C leaves: (inner, outer) are its C coordinates
// along the contiguous and the row dimension.
__device__ __forceinline__ void store_block(const CUtensorMap* map, const void* blk, const EpiParams& ep, int inner,
                                            int outer, int cz, int bz) {
    if (ep.c_split) {
        const int lo = inner % ep.c_split, hi = inner / ep.c_split;
        if (ep.mode == EPI_ASSIGN) tma_store_5d(map, blk, lo, hi, outer, cz, bz);
        else tma_reduce_add_5d(map, blk, lo, hi, outer, cz, bz);
    } else {
        if (ep.mode == EPI_ASSIGN) tma_store_4d(map, blk, inner, outer, cz, bz);
        else tma_reduce_add_4d(map, blk, inner, outer, cz, bz);
    }
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most N committed bulk groups may still be reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Programmatic dependent launch: wait for the preceding kernel's writes,
// then let the following kernel start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// UMMA shared-memory descriptor (sm100 version bits).  Layout types:
// 2 = 128-byte swizzle with 16-byte atoms (K-major operands),
// 1 = 128-byte swizzle with 32-byte atoms, the only MN-major layout the
//     tensor cores accept for 32-bit (tf32) elements.
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Atom32 = 1;

__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint32_t layout = kLayoutSW128) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm100)
    d |= (uint64_t)(layout & 7u) << 61;
    return d;
}

// Operand tile descriptors for k-step kk (8 tf32 of K) of a k-block:
//  K-major : rows of 128 B (32 K-values), 8-row swizzle atoms 1024 B apart;
//            a k-step advances 32 B along the row.
//  MN-major: 32 K-rows x 128 B (32 MN-values) per k-block and 32-column
//            chunk, chunks `lbo` bytes apart along MN (4096 B, or 4096 B
//            per k-block of a stage); 32-byte-atom swizzle repeats every 4
//            rows (SBO = 512 B); a k-step advances 8 rows = 1024 B.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) { return make_sdesc(base + kk * 32, 16, 1024); }
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk, uint32_t lbo = 4096) {
    return make_sdesc(base + kk * 1024, lbo, 512, kLayoutSW128Atom32);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}

// ------------------------- CTA pairs (cta_group::2) -------------------------
// A pair of CTAs (a 2-CTA cluster) computes one 256-row tile: each CTA
// stages its 128 rows of A and half of the tile's B columns at the same
// shared-memory offsets; the even CTA issues 256 x BN MMAs that read both
// CTAs' stages and write each CTA's 128 accumulator rows into its own TMEM.
// Both CTAs' copies complete on the even CTA's full barrier; its commits
// arrive on both CTAs' barriers; both epilogues release the accumulator on
// the even CTA's barrier.  No load uses cluster multicast.

// shared::cluster address of the same shared-memory offset in CTA 0 of the cluster
__device__ __forceinline__ uint32_t rank0_addr(const void* p) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
    return r;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// tiled load whose completion is counted on an mbarrier of either CTA of the pair
__device__ __forceinline__ void tma_load_4d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int c0,
                                                 int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int c0,
                                                 int c1, int c2, int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accum) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(z)
        : "memory");
}

// arrives once on the barrier at this offset in both CTAs of the pair when
// the issuing thread's MMAs retire
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// A stage holds KPL k-blocks of A (and of B): K-major [kb][rows][32 K],
// MN-major [32-column chunk][kb][32 K rows][32 MN].
template <int BN, int STAGES, int KPL = 1>
struct Smem {
    static constexpr int A_BYTES = KPL * BM * BK * 4;  // 16 KB per k-block
    static constexpr int B_BYTES = KPL * BN * BK * 4;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
    static constexpr int EPI_WARP_BYTES = 2 * 32 * 32 * 4;  // two 4 KB blocks (>= 32 x kEpiLd floats)
    static constexpr int BAR_OFFSET = EPI_OFFSET + kEpiWarps * EPI_WARP_BYTES;
    // full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], drain, consumed[STAGES]
    static constexpr int N_BARS = 3 * STAGES + 5;
    static constexpr int TOTAL = BAR_OFFSET + N_BARS * 8 + 16 + 1024;  // + TMEM slot, abort flag, alignment
};

// A_MN: A is stored MN-major ([K][M]); B_MN: B is stored MN-major ([K][N]).
// PAIR: launched as 2-CTA clusters; a tile is 256 x BN (cta_group::2 MMAs),
// each CTA staging 128 rows of A and BN/2 columns of B.
// KPL: k-blocks per stage, each operand's stage arriving as one copy of
// the split view (KPL = 2 only for operands that have one).
template <bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR = false, int KPL = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ GemmGroup grp) {
    constexpr int BNC = PAIR ? BN / 2 : BN;  // B columns staged by this CTA
    constexpr int BMT = PAIR ? 2 * BM : BM;  // tile rows
    using L = Smem<BNC, STAGES, KPL>;
    static_assert(L::EPI_WARP_BYTES >= 32 * kEpiLd * 4, "staging");
    static_assert(BNC % 32 == 0, "B staged in 32-column boxes");
    constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators (this CTA's 128 rows x BN)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* consumed = drain + 1;  // a stage's MMAs retired (column sums read it then)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(consumed + STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t total_tiles = grp.tile_start[grp.n];

    if (threadIdx.x == 0) {
        // a stage is released by the MMA commit, and by each epilogue warp
        // too when they sum B's columns (after the commit on consumed[s])
        const bool follow = B_MN && grp.colsum;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], follow ? 1 + kEpiWarps : 1);
            mbar_init(&consumed[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int g = 0; g < (grp.kcat > grp.n ? grp.kcat : grp.n); ++g) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&grp.a[g])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&grp.b[g])) : "memory");
            if (grp.ep[g].tma_epi)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&grp.c[g])) : "memory");
        }
    }
    if (warp == 0) {
        if constexpr (PAIR) {
            // collective over the same warp of both CTAs
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    // the peer's barriers are initialised before any copy or commit reaches them
    if constexpr (PAIR) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int rank = PAIR ? (int)cluster_rank() : 0;
    const int64_t t_first = PAIR ? blockIdx.x / 2 : blockIdx.x;
    const int64_t t_step = PAIR ? gridDim.x / 2 : gridDim.x;
    // everything above overlapped the previous kernel; its outputs are read
    // (and C written) only from here on
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            uint32_t last_parity[STAGES];
            bool issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = false;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t t = t_first; ok && t < total_tiles; t += t_step) {
                int64_t tl;
                const int g = locate(grp, t, tl);
                // a register copy: a reference into the parameter space would be
                // re-read after every shared-memory or global access
                const EpiParams ep = grp.ep[g];
                const CUtensorMap* tmA = &grp.a[g];
                const CUtensorMap* tmB = &grp.b[g];
                const Tile x = tile_at(ep, tl, BN, BMT);
                const int a_c = ep.a_has_c ? x.cidx : 0, a_b = ep.a_has_b ? x.bidx : 0;
                const int b_c = ep.b_has_c ? x.cidx : 0, b_b = ep.b_has_b ? x.bidx : 0;
                for (int i = 0; i < x.nkb; i += KPL) {
                    if (!wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + s * L::STAGE_BYTES;
                    uint8_t* sb = sa + L::A_BYTES;
                    const int k0 = (x.kb_begin + i) * BK;
                    // this CTA's rows of A and columns of B
                    const int mo = x.m0 + rank * BM, no = x.n0 + rank * BNC;
                    // a pair's copies all complete on CTA 0's barrier, which
                    // expects both CTAs' bytes
                    const uint32_t bar = PAIR ? rank0_addr(&full[s]) : 0u;
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(PAIR ? 2 : 1) * L::STAGE_BYTES);
                    auto load = [&](const CUtensorMap* map, void* dst, int c0, int c1, int c2, int c3) {
                        if constexpr (PAIR) tma_load_4d_pair(map, bar, dst, c0, c1, c2, c3);
                        else tma_load_4d(map, &full[s], dst, c0, c1, c2, c3);
                    };
                    auto load5 = [&](const CUtensorMap* map, void* dst, int c1, int c2, int c3, int c4) {
                        if constexpr (PAIR) tma_load_5d_pair(map, bar, dst, 0, c1, c2, c3, c4);
                        else tma_load_5d(map, &full[s], dst, 0, c1, c2, c3, c4);
                    };
                    if (KPL == 1 && !A_MN && B_MN && ep.conv == 1) {
                        // weights [tap][m][c]; the pixels of a tap are the output
                        // pixels moved by whole rows in the flattened image plane
                        const int kb = x.kb_begin + i;
                        const int tap = kb / ep.cv_cblk, c0 = (kb - tap * ep.cv_cblk) * BK;
                        const int kh = tap / ep.cv_kw, kw = tap - kh * ep.cv_kw;
                        const int zc = kw * ep.cv_nb + x.bidx;
                        const int dp = (kh - ep.cv_pad) * ep.cv_w;
                        load(tmA, sa, c0, mo, tap, 0);
#pragma unroll
                        for (int j = 0; j < BNC / 32; ++j) load(tmB, sb + j * 4096, no + 32 * j + dp, c0, zc, 0);
                    } else if (KPL == 1 && A_MN && !B_MN && ep.conv == 3) {
                        const int kb = x.kb_begin + i;
                        const int tap = kb / ep.cv_cblk, c0 = (kb - tap * ep.cv_cblk) * BK;
                        const int kh = tap / ep.cv_kw, kw = tap - kh * ep.cv_kw;
                        const int zc = kw * ep.cv_nb + x.bidx;
                        const int dp = (kh - ep.cv_pad) * ep.cv_w;
#pragma unroll
                        for (int j = 0; j < BM / 32; ++j) load(tmA, sa + j * 4096, mo + 32 * j + dp, c0, zc, 0);
                        load(tmB, sb, c0, no, tap, 0);
                    } else if (KPL == 1 && !A_MN && !B_MN && ep.conv == 2) {
                        // B rows = channels no.. of tap x.cidx at pixels k0..k0+31
                        const int kh = x.cidx / ep.cv_kw, kw = x.cidx - kh * ep.cv_kw;
                        load(tmA, sa, k0, mo, a_c, a_b);
                        load(tmB, sb, k0 + (kh - ep.cv_pad) * ep.cv_w, no, kw * ep.cv_nb + x.bidx, 0);
                    } else {
                        // the segment of a concatenated reduction this
                        // stage reads (a stage never straddles two)
                        const CUtensorMap* mA = tmA;
                        const CUtensorMap* mB = tmB;
                        int kc = k0, asp = ep.a_split, bsp = ep.b_split;
                        if (grp.kcat > 1) {
                            const int kb = x.kb_begin + i;
                            int gk = 0;
                            while (gk + 1 < grp.kcat && kb >= grp.kcat_kb[gk + 1]) ++gk;
                            mA = &grp.a[gk];
                            mB = &grp.b[gk];
                            kc = (kb - grp.kcat_kb[gk]) * BK;
                            asp = grp.ep[gk].a_split;
                            bsp = grp.ep[gk].b_split;
                        }
                        // split views: the stage's KPL k-blocks of all its
                        // rows (K-major) or 32-column chunks (MN-major) in
                        // one copy per operand
                        if (asp) {
                            if (A_MN) load5(mA, sa, kc, mo >> 5, a_c, a_b);
                            else load5(mA, sa, mo, kc >> 5, a_c, a_b);
                        } else if (A_MN) {
#pragma unroll
                            for (int j = 0; j < BM / 32; ++j) load(mA, sa + j * 4096, mo + 32 * j, kc, a_c, a_b);
                        } else {
                            load(mA, sa, kc, mo, a_c, a_b);
                        }
                        if (bsp) {
                            if (B_MN) load5(mB, sb, kc, no >> 5, b_c, b_b);
                            else load5(mB, sb, no, kc >> 5, b_c, b_b);
                        } else if (B_MN) {
#pragma unroll
                            for (int j = 0; j < BNC / 32; ++j) load(mB, sb + j * 4096, no + 32 * j, kc, b_c, b_b);
                        } else {
                            load(mB, sb, kc, no, b_c, b_b);
                        }
                    }
                    issued[s] = true;
                    last_parity[s] = ph;
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            // on abort, let issued copies land before the CTA leaves (in a
            // pair they complete on CTA 0's barriers, which CTA 0 drains)
            if (*abort_flag && rank == 0) {
                for (int u = 0; u < STAGES; ++u)
                    if (issued[u]) drain_wait(&full[u], last_parity[u]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ------------------------------- MMA issuer -------------------------------
            // (in a pair only CTA 0 issues: 256 x BN MMAs over both CTAs' stages)
            // instruction descriptor: D=f32, A=B=tf32, transpose bits, N>>3, M>>4
            const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) |
                                   ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                                   ((uint32_t)(BMT >> 4) << 24);
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int acc = 0;
            for (int64_t t = t_first; ok && t < total_tiles; t += t_step, ++acc) {
                int64_t tl;
                const int g = locate(grp, t, tl);
                const EpiParams ep = grp.ep[g];
                const Tile x = tile_at(ep, tl, BN, BMT);
                const int buf = acc & 1;
                const uint32_t use = (uint32_t)(acc >> 1);
                if (!wait_bounded(&tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(buf * BN);
                for (int i = 0; i < x.nkb; i += KPL) {
                    if (!wait_bounded(&full[s], ph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * L::STAGE_BYTES);
                    const uint32_t sb = sa + L::A_BYTES;
                    // the stage's last copy may reach past the tile's k-range
                    const int nv = min(KPL, x.nkb - i);
                    for (int kb = 0; kb < nv; ++kb) {
                        const uint32_t ka = A_MN ? sa + kb * 4096 : sa + kb * (BM * BK * 4);
                        const uint32_t kbb = B_MN ? sb + kb * 4096 : sb + kb * (BNC * BK * 4);
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            const uint64_t ad = A_MN ? mnmajor_desc(ka, kk, KPL * 4096) : kmajor_desc(ka, kk);
                            const uint64_t bd = B_MN ? mnmajor_desc(kbb, kk, KPL * 4096) : kmajor_desc(kbb, kk);
                            const uint32_t accum = (i > 0 || kb > 0 || kk > 0) ? 1u : 0u;
                            if constexpr (PAIR) mma_tf32_pair(tmem_d, ad, bd, idesc, accum);
                            else mma_tf32(tmem_d, ad, bd, idesc, accum);
                        }
                    }
                    if constexpr (PAIR) mma_commit_pair_both(&empty[s]);
                    else mma_commit(&empty[s]);
                    if (B_MN && grp.colsum) {
                        if constexpr (PAIR) mma_commit_pair_both(&consumed[s]);
                        else mma_commit(&consumed[s]);
                    }
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                // arrives once every MMA of this tile retired
                if constexpr (PAIR) mma_commit_pair_both(&tmem_full[buf]);
                else mma_commit(&tmem_full[buf]);
            }
            // every MMA issued above retires before TMEM is released
            if constexpr (PAIR) mma_commit_pair_local(drain);
            else mma_commit(drain);
            drain_wait(drain, 0);
        }
        __syncwarp();
    } else {
        // --------------------------------- epilogue ---------------------------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        float* stage = reinterpret_cast<float*>(smem + L::EPI_OFFSET + (warp - 2) * L::EPI_WARP_BYTES);
        const int rsub = lane >> 3, c4 = (lane & 7) * 4;
        int acc = 0;
        uint32_t blocks_out = 0;  // bulk groups this warp committed
        int es = 0;               // the stage ring as the MMA issuer walks it (column sums)
        uint32_t eph = 0;
        for (int64_t t = t_first; t < total_tiles; t += t_step, ++acc) {
            int64_t tl;
            const int g = locate(grp, t, tl);
            const EpiParams ep = grp.ep[g];  // register copy (see the producer)
            const CUtensorMap* tmC = &grp.c[g];
            const Tile x = tile_at(ep, tl, BN, BMT);
            const int buf = acc & 1;
            const uint32_t use = (uint32_t)(acc >> 1);
            if constexpr (B_MN) {
                if (grp.colsum) {
                    // B's columns summed over the tile's k-range while its stages
                    // pass: 32-column chunk ch of a stage holds KPL k-blocks of 32
                    // rows of 128 bytes (one k each), swizzled in 32-byte units
                    // (the MN-major 128-byte swizzle with 32-byte atoms): unit j of
                    // row r sits at j ^ (r % 4); lane l sums column ch * 32 + l.
                    // A stage is read once its MMAs retired (consumed[s], which the
                    // MMA issuer commits in both CTAs of a pair, each summing the
                    // columns it staged) and released here (its empty barrier
                    // expects these warps), summed or not.
                    constexpr int kCh = (BNC / 32 + kEpiWarps - 1) / kEpiWarps;
                    const bool sum_here = ep.colsum != nullptr && x.m0 == 0;
                    const int e = warp - 2;
                    float cs[kCh];
#pragma unroll
                    for (int u = 0; u < kCh; ++u) cs[u] = 0.0f;
                    bool ok = true;
                    for (int i = 0; i < x.nkb; i += KPL) {
                        ok = __all_sync(0xffffffffu, wait_bounded(&consumed[es], eph, abort_flag));
                        if (!ok) break;
                        if (sum_here) {
                            const uint8_t* sb = smem + es * L::STAGE_BYTES + L::A_BYTES;
                            const int nv = min(KPL, x.nkb - i);
#pragma unroll
                            for (int u = 0; u < kCh; ++u) {
                                const int ch = e + u * kEpiWarps;
                                if (ch >= BNC / 32) break;
                                for (int kb = 0; kb < nv; ++kb) {
                                    const uint8_t* blk = sb + ch * (KPL * 4096) + kb * 4096 + (lane & 7) * 4;
#pragma unroll 8
                                    for (int r = 0; r < 32; ++r)
                                        cs[u] += *reinterpret_cast<const float*>(
                                            blk + r * 128 + ((((lane >> 3) ^ (r & 3))) << 5));
                                }
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[es]);
                        if (++es == STAGES) {
                            es = 0;
                            eph ^= 1u;
                        }
                    }
                    if (!ok) break;
                    if (sum_here && x.nkb > 0) {
#pragma unroll
                        for (int u = 0; u < kCh; ++u) {
                            const int ch = e + u * kEpiWarps;
                            const int col = x.n0 + rank * BNC + ch * 32 + lane;
                            if (ch < BNC / 32 && col < ep.N) atomicAdd(ep.colsum + col, cs[u]);
                        }
                    }
                }
            }
            // the tcgen05.ld below is warp-collective: leave the loop together
            const bool ready = wait_bounded(&tmem_full[buf], use & 1u, abort_flag);
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            float* Cbase = ep.C + (int64_t)x.bidx * ep.c_stride_b + (int64_t)x.cidx * ep.c_stride_c;
            const bool live = x.nkb > 0;
            // the warp-store path's bias for this lane's 4 columns of block cc,
            // loaded one block ahead so its latency hides behind the stores
            const bool row_bias = ep.bias && x.kb_begin == 0 && !ep.tma_epi;  // split 0 adds the bias
            auto bias4 = [&](int col) {
                float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
                if (!row_bias) return b;
                if (ep.vec && col + 4 <= ep.N) return __ldg(reinterpret_cast<const float4*>(ep.bias + col));
                if (col < ep.N) b.x = __ldg(ep.bias + col);
                if (col + 1 < ep.N) b.y = __ldg(ep.bias + col + 1);
                if (col + 2 < ep.N) b.z = __ldg(ep.bias + col + 2);
                if (col + 3 < ep.N) b.w = __ldg(ep.bias + col + 3);
                return b;
            };
            float4 bias_next = bias4(x.n0 + c4);
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc) {
                const int col0 = x.n0 + cc * 32;
                if (col0 >= ep.N) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + cc * 32), r);
                const float4 bias_cur = bias_next;
                if (cc + 1 < BN / 32) bias_next = bias4(col0 + 32 + c4);
                if (!live) continue;
                if (ep.tma_epi) {
                    const int row0 = x.m0 + rank * BM + q * 32;
                    if (row0 >= ep.M) continue;  // warp-uniform: this quarter lies below the matrix
                    float* blk = stage + (blocks_out & 1u) * 1024;
                    if (blocks_out >= 2) {
                        if (lane == 0) bulk_wait_read<1>();
                        __syncwarp();
                    }
                    if (ep.c_trans) {
                        // C stores the tile transposed: block row j (C row col0 + j)
                        // holds the 32 tile rows, lane's word in chunk
                        // (lane / 4) ^ (j % 8) (128-byte swizzle); the bias is per
                        // tile column
                        const bool add_bias = ep.bias && x.kb_begin == 0;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            float v = ep.alpha * __uint_as_float(r[j]);
                            if (add_bias && col0 + j < ep.N) v += __ldg(ep.bias + col0 + j);
                            blk[j * 32 + ((((lane >> 2) ^ (j & 7))) << 2) + (lane & 3)] = v;
                        }
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            store_block(tmC, blk, ep, row0, col0, ep.c_has_c ? x.cidx : 0, ep.c_has_b ? x.bidx : 0);
                            bulk_commit();
                        }
                        ++blocks_out;
                        continue;
                    }
                    // row `lane` of the block: alpha * acc + bias, 16-byte chunk j
                    // stored at chunk j ^ (row % 8) (128-byte swizzle)
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float4 v = make_float4(ep.alpha * __uint_as_float(r[4 * j]),
                                               ep.alpha * __uint_as_float(r[4 * j + 1]),
                                               ep.alpha * __uint_as_float(r[4 * j + 2]),
                                               ep.alpha * __uint_as_float(r[4 * j + 3]));
                        if (ep.bias && x.kb_begin == 0) {  // split 0 adds the bias
                            const int cb = col0 + 4 * j;
                            if (ep.vec && cb + 4 <= ep.N) {
                                const float4 b = *reinterpret_cast<const float4*>(ep.bias + cb);
                                v.x += b.x;
                                v.y += b.y;
                                v.z += b.z;
                                v.w += b.w;
                            } else {
                                if (cb < ep.N) v.x += ep.bias[cb];
                                if (cb + 1 < ep.N) v.y += ep.bias[cb + 1];
                                if (cb + 2 < ep.N) v.z += ep.bias[cb + 2];
                                if (cb + 3 < ep.N) v.w += ep.bias[cb + 3];
                            }
                        }
                        *reinterpret_cast<float4*>(blk + lane * 32 + ((j ^ (lane & 7)) * 4)) = v;
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        store_block(tmC, blk, ep, col0, row0, ep.c_has_c ? x.cidx : 0, ep.c_has_b ? x.bidx : 0);
                        bulk_commit();
                    }
                    ++blocks_out;
                    continue;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<float4*>(stage + lane * kEpiLd + 4 * j) =
                        make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                    __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                __syncwarp();
                const int col = col0 + c4;
                const bool vec = ep.vec && col + 4 <= ep.N;
                const float4 bv = bias_cur;
                // every staged value first, then the stores: a store through a
                // generic pointer could alias the staging area, so loads after
                // it would wait for it
                float4 staged[8];
#pragma unroll
                for (int it = 0; it < 8; ++it)
                    staged[it] = *reinterpret_cast<const float4*>(stage + (it * 4 + rsub) * kEpiLd + c4);
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    const int rr = it * 4 + rsub;
                    const int row = x.m0 + rank * BM + q * 32 + rr;
                    if (row >= ep.M || col >= ep.N) continue;
                    float4 v = staged[it];
                    v.x = ep.alpha * v.x + bv.x;
                    v.y = ep.alpha * v.y + bv.y;
                    v.z = ep.alpha * v.z + bv.z;
                    v.w = ep.alpha * v.w + bv.w;
                    float* crow = Cbase + (int64_t)row * ep.ldc;
                    if (vec) {
                        float4* dst = reinterpret_cast<float4*>(crow + col);
                        if (ep.mode == EPI_ASSIGN) {
                            *dst = v;
                        } else if (ep.mode == EPI_ACCUM) {
                            float4 o = *dst;
                            o.x += v.x;
                            o.y += v.y;
                            o.z += v.z;
                            o.w += v.w;
                            *dst = o;
                        } else {
                            atomicAdd(dst, v);
                        }
                    } else {
                        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            if (col + u >= ep.N) break;
                            if (ep.mode == EPI_ASSIGN) crow[col + u] = e[u];
                            else if (ep.mode == EPI_ACCUM) crow[col + u] += e[u];
                            else atomicAdd(crow + col + u, e[u]);
                        }
                    }
                }
                __syncwarp();
            }
            // this accumulator may be overwritten once every lane's loads retired
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(rank0_addr(&tmem_empty[buf]));
                else mbar_arrive(&tmem_empty[buf]);
            }
        }
        // bulk stores must finish reading shared memory (and land) before exit
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    // a pair leaves together: CTA 0's MMAs (drained above) read this CTA's
    // stages and write its TMEM, and its epilogue arrivals target CTA 0
    if constexpr (PAIR) cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                         : "memory");
    }
}

// ---------------------------------------------------------------------------
// Attention scores with the column softmax, keys on the TMEM lanes.
//
// The reference normalises each key column of the scores over the queries
// (SOFTMAX / SOFTMASK type 1, Engine/kernels.cu:2134-2235) and backs it up
// with the per-column dot product (deriv_softmax, :2149-2181).  Computing
// the transposed product S^T = K Q^T puts one key on each TMEM lane and all
// its queries along the lane's columns, so a column belongs to the QG warps
// that read one TMEM lane quarter (each takes SQ / QG of the queries): the
// max, the sum and the dot product are thread-local loops plus one exchange
// of partials through shared memory, and the scores never reach HBM.  One
// CTA of 4 * QG warps per (batch, head, block of 128 keys), two per SM (one
// CTA's operand loads and products overlap the other's epilogue):
//   MODE 0  S^T = scale * K_blk Q^T -> P[b,h,:,keys] = column softmax
//           (causal: key > query contributes 0; the max runs over every
//           query, as the reference's SoftMask takes it)
//   MODE 1  dP^T = V_blk dO^T, then with P read back per column,
//           dS = P (dP - sum_q P dP) -> out[b,h,:,keys]
// Operands (HD columns of every row) arrive by TMA as K-major tiles (128-byte
// swizzle, 32 floats per k-block); the product is tcgen05.mma kind::tf32,
// M = 128 keys, N = SQ queries, into SQ TMEM columns.  Stores and the P
// reads of MODE 1 run along the keys: a warp touches 32 consecutive floats
// of one query row.
struct AttnKeysParams {
    CUtensorMap a_map;  // keys:    (HD, S_k, H, B) view of K (MODE 0) or V (MODE 1)
    CUtensorMap b_map;  // queries: (HD, S_q, H, B) view of Q (MODE 0) or dO (MODE 1)
    const float* P;     // MODE 1: probabilities [B, H, Sq, Sk]
    float* out;         // P (MODE 0; may be null) or dS (MODE 1), [B, H, Sq, Sk]
    float* stats;       // MODE 0, optional: column max [B*H*Sk] then inverse column sum [B*H*Sk]
    int H, Sq, Sk, key_blocks;
    float scale;
    int causal;
};

constexpr float kLog2e = 1.4426950408889634f;

// 2^x with the PTX approximate instruction (relative error around 2^-22,
// far below the tf32 rounding the probabilities take before their
// products; subnormal results flush to 0)
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD, int SQ>
struct AttnKeysSmem {
    static constexpr int KB = HD / 32;
    static constexpr int A_BYTES = 128 * 128;  // one k-block of 128 key rows
    static constexpr int B_BYTES = SQ * 128;   // one k-block of SQ query rows
    static constexpr int B_OFFSET = KB * A_BYTES;
    static constexpr int BAR_OFFSET = B_OFFSET + KB * B_BYTES;
    static constexpr int TOTAL = BAR_OFFSET + 64 + 4 * 128 * 4 + 1024;  // barriers, TMEM slot, abort flag,
                                                                        // per-key partials; alignment
};

// query groups per key: the warps that share a TMEM lane quarter split the
// queries (4 for the softmax, whose registers allow 512 threads at two CTAs
// per SM; 2 for the score gradient, which keeps two P chunks in registers)
template <int MODE>
constexpr int attn_keys_groups() {
    return MODE == 0 ? 4 : 2;
}

template <int MODE, int HD, int SQ>
__global__ void __launch_bounds__(128 * attn_keys_groups<MODE>(), 2)
    attn_keys_kernel(const __grid_constant__ AttnKeysParams p) {
    constexpr int QG = attn_keys_groups<MODE>();
    using L = AttnKeysSmem<HD, SQ>;
    constexpr int KB = L::KB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
    uint64_t* done = full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblk = blockIdx.x % p.key_blocks;
    const int bh = blockIdx.x / p.key_blocks;
    const int h = bh % p.H, b = bh / p.H;
    const int key0 = kblk * 128;

    if (threadIdx.x == 0) {
        mbar_init(full, 1);
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.a_map)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.b_map)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)SQ)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the previous kernel's outputs are read only from here on; the next
    // kernel may be scheduled once every CTA of this grid holds its TMEM
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    bool mma_issued = false;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(full, (uint32_t)(KB * (L::A_BYTES + L::B_BYTES)));
#pragma unroll
        for (int kk = 0; kk < KB; ++kk) {
            tma_load_4d(&p.a_map, full, smem + kk * L::A_BYTES, 32 * kk, key0, h, b);
            tma_load_4d(&p.b_map, full, smem + L::B_OFFSET + kk * L::B_BYTES, 32 * kk, 0, h, b);
        }
        if (wait_bounded(full, 0, abort_flag)) {
            tc_fence_after();
            // D = f32, A = B = tf32, both K-major, N = SQ, M = 128
            const uint32_t idesc =
                (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(SQ >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
#pragma unroll
            for (int kk = 0; kk < KB; ++kk) {
                const uint32_t sa = smem_u32(smem + kk * L::A_BYTES);
                const uint32_t sb = smem_u32(smem + L::B_OFFSET + kk * L::B_BYTES);
#pragma unroll
                for (int k8 = 0; k8 < 4; ++k8)
                    mma_tf32(tmem, kmajor_desc(sa, k8), kmajor_desc(sb, k8), idesc, (kk | k8) ? 1u : 0u);
            }
            mma_commit(done);
            mma_issued = true;
        } else {
            drain_wait(full, 0);  // the copies land before the CTA leaves
        }
    }
    // every thread takes the same branch: the epilogue exchanges per-key
    // partials through shared memory between the two warps of a lane quarter
    const bool issued = __syncthreads_or(mma_issued ? 1 : 0) != 0;
    const bool ready = __syncthreads_and((issued && wait_bounded(done, 0, abort_flag)) ? 1 : 0) != 0;
    if (ready) {
        tc_fence_after();
        // warp w reads TMEM lanes 32 (w % 4).. (its keys) and the columns of
        // query group w / 4
        constexpr int HALF = SQ / QG;  // queries per group
        float* red = reinterpret_cast<float*>(smem + L::BAR_OFFSET + 64);  // [QG][128] partials
        const int kl = (warp & 3) * 32 + lane, half = warp >> 2;
        const int key = key0 + kl;
        const bool live = key < p.Sk;
        const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(half * HALF);
        const int64_t base = (int64_t)bh * p.Sq * p.Sk + key;
        const int q0 = half * HALF;
        uint32_t r[32];
        if (MODE == 0) {
            float m = -FLT_MAX;
            for (int c = 0; c < HALF / 32; ++c) {
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (q0 + c * 32 + j < p.Sq) m = fmaxf(m, p.scale * __uint_as_float(r[j]));
            }
            red[half * 128 + kl] = m;
            __syncthreads();
            m = red[kl];
#pragma unroll
            for (int g = 1; g < QG; ++g) m = fmaxf(m, red[g * 128 + kl]);
            __syncthreads();
            // exp(scale s - m) = exp2(s c2 - m log2 e)
            const float c2 = p.scale * kLog2e, m2 = m * kLog2e;
            float sum = 0.f;
            for (int c = 0; c < HALF / 32; ++c) {
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int q = q0 + c * 32 + j;
                    if (q < p.Sq && !(p.causal && key > q)) sum += exp2_approx(fmaf(__uint_as_float(r[j]), c2, -m2));
                }
            }
            red[half * 128 + kl] = sum;
            __syncthreads();
            sum = red[kl];
#pragma unroll
            for (int g = 1; g < QG; ++g) sum += red[g * 128 + kl];
            const float inv = 1.0f / (sum < 1e-45f ? 1.0f : sum);
            if (p.stats && live && half == 0) {
                const int64_t nk = (int64_t)gridDim.x / p.key_blocks * p.Sk;  // B * H * Sk
                p.stats[(int64_t)bh * p.Sk + key] = m;
                p.stats[nk + (int64_t)bh * p.Sk + key] = inv;
            }
            for (int c = 0; p.out && c < HALF / 32; ++c) {
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
                if (live) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int q = q0 + c * 32 + j;
                        const float e =
                            (p.causal && key > q) ? 0.f : exp2_approx(fmaf(__uint_as_float(r[j]), c2, -m2));
                        if (q < p.Sq) p.out[base + (int64_t)q * p.Sk] = e * inv;
                    }
                }
            }
        } else {
            // P of this thread's key column, one chunk of 32 queries ahead:
            // the loads of chunk c + 1 are in flight while chunk c's dP
            // comes out of TMEM and is consumed
            float pc[32], pn[32];
            auto load_p = [&](float(&dst)[32], int c) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int q = q0 + c * 32 + j;
                    dst[j] = (live && q < p.Sq) ? __ldg(p.P + base + (int64_t)q * p.Sk) : 0.f;
                }
            };
            float d = 0.f;
            load_p(pn, 0);
            for (int c = 0; c < HALF / 32; ++c) {
#pragma unroll
                for (int j = 0; j < 32; ++j) pc[j] = pn[j];
                if (c + 1 < HALF / 32) load_p(pn, c + 1);
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
#pragma unroll
                for (int j = 0; j < 32; ++j) d += pc[j] * __uint_as_float(r[j]);
            }
            red[half * 128 + kl] = d;
            __syncthreads();
            d = red[kl];
#pragma unroll
            for (int g = 1; g < QG; ++g) d += red[g * 128 + kl];
            load_p(pn, 0);
            for (int c = 0; c < HALF / 32; ++c) {
#pragma unroll
                for (int j = 0; j < 32; ++j) pc[j] = pn[j];
                if (c + 1 < HALF / 32) load_p(pn, c + 1);
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
                if (live) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int q = q0 + c * 32 + j;
                        if (q < p.Sq) p.out[base + (int64_t)q * p.Sk] = pc[j] * (__uint_as_float(r[j]) - d);
                    }
                }
            }
        }
    } else if (threadIdx.x == 0 && mma_issued) {
        drain_wait(done, 0);  // the MMAs retire before TMEM is released
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)SQ)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no libcuda link)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Operand view: element (inner i, outer o, channel c, batch b) lives at
// base + i + o*ld + c*sc + b*sb.  Extents of broadcast dims are 1.
struct OperandView {
    const float* base;
    int64_t inner, outer, nc, nb;
    int64_t ld, sc, sb;  // elements
};

// K-major tiles use the 16-byte-atom 128-byte swizzle; MN-major tiles the
// 32-byte-atom one, matching the UMMA layout types above.
static bool encode_operand(CUtensorMap* map, const OperandView& v, int box_inner, int box_outer,
                           bool mn_major = false, CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)v.inner, (cuuint64_t)v.outer, (cuuint64_t)v.nc, (cuuint64_t)v.nb};
    // byte strides of dims 1..3 (must be multiples of 16 and non-zero)
    int64_t sc = v.sc, sb = v.sb;
    if (v.nc == 1) sc = v.ld * v.outer;
    if (v.nb == 1) sb = (v.nc == 1 ? v.ld * v.outer : sc * v.nc);
    cuuint64_t strides[3] = {(cuuint64_t)(v.ld * 4), (cuuint64_t)(sc * 4), (cuuint64_t)(sb * 4)};
    cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, dt, 4, const_cast<float*>(v.base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Split view of an operand whose contiguous extent is a multiple of 32:
// (32, outer, inner / 32, channel, batch), so one copy brings a stage.
// K-major (inner = K): box (32, rows, kpl) lands as [kb][rows][32 K];
// MN-major (inner = M or N): box (32, 32 * kpl, mn / 32) lands as
// [32-column chunk][32 * kpl K rows][32 MN].
static bool encode_operand_split(CUtensorMap* map, const OperandView& v, bool mn_major, int box_rows, int kpl,
                                 CUtensorMapDataType dt) {
    EncodeTiledFn enc = get_encode();
    if (!enc || v.inner % 32 != 0 || box_rows % 32 != 0) return false;
    int64_t sc = v.sc, sb = v.sb;
    if (v.nc == 1) sc = v.ld * v.outer;
    if (v.nb == 1) sb = (v.nc == 1 ? v.ld * v.outer : sc * v.nc);
    cuuint64_t dims[5] = {32, (cuuint64_t)v.outer, (cuuint64_t)(v.inner / 32), (cuuint64_t)v.nc, (cuuint64_t)v.nb};
    cuuint64_t strides[4] = {(cuuint64_t)(v.ld * 4), 128, (cuuint64_t)(sc * 4), (cuuint64_t)(sb * 4)};
    cuuint32_t box[5] = {32, (cuuint32_t)(mn_major ? 32 * kpl : box_rows), (cuuint32_t)(mn_major ? box_rows / 32 : kpl),
                         1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(map, dt, 5, const_cast<float*>(v.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 tensor map of `rank` (4 or 5) dims with explicit extents, element
// strides of dims 1.. and box.
static bool encode_map(CUtensorMap* map, const float* base, const int64_t* dims, const int64_t* strides,
                       const int* box, CUtensorMapSwizzle swizzle, int rank = 4,
                       CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32) {
    EncodeTiledFn enc = get_encode();
    if (!enc || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], e[5] = {1, 1, 1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = (cuuint64_t)dims[i];
        b[i] = (cuuint32_t)box[i];
    }
    for (int i = 0; i + 1 < rank; ++i) st[i] = (cuuint64_t)(strides[i] * 4);
    return enc(map, dt, (cuuint32_t)rank, const_cast<float*>(base), d, st, b, e,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR = false, int KPL = 1>
static int launch_tc(const GemmGroup& grp, cudaStream_t st) {
    using L = Smem<PAIR ? BN / 2 : BN, STAGES, KPL>;
    static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
    static_assert(sizeof(GemmGroup) <= 4000, "kernel parameter space");
    auto kern = gemm_tf32_kernel<A_MN, B_MN, BN, STAGES, PAIR, KPL>;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) != cudaSuccess)
            return launch_status();
        configured = true;
    }
    // persistent: one CTA (or CTA pair) per SM (pair); the shared-memory
    // ring admits one per SM; the prologue may overlap the previous kernel
    // (programmatic dependent launch)
    const int64_t tiles = grp.tile_start[grp.n];
    int64_t units = kSMs;
    if constexpr (PAIR) {
        // as many pairs as can be resident at once (clusters need both SMs of
        // a pair free in one GPC)
        static int max_pairs = 0;
        if (max_pairs == 0) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3(kSMs);
            q.blockDim = dim3(kThreads);
            q.dynamicSmemBytes = L::TOTAL;
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = 2;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.attrs = qa;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = kSMs / 2;
            }
            max_pairs = n < kSMs / 2 ? n : kSMs / 2;
        }
        units = max_pairs;
    }
    const int grid = (int)(tiles < units ? tiles : units) * (PAIR ? 2 : 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = PAIR ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, kern, grp) != cudaSuccess) return launch_status();
    return launch_status();
}

}  // namespace tc

static bool tc_eligible(const GemmProblem& p) {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (!al(p.A) || !al(p.B)) return false;
    if ((p.lda & 3) || (p.ldb & 3)) return false;
    if ((p.a_sb & 3) || (p.a_sc & 3) || (p.b_sb & 3) || (p.b_sc & 3)) return false;
    // N tiles of >= 64 columns: tiny N (e.g. 10 logits) goes to the SIMT path.
    if (p.N < 32 || p.M < 16) return false;
    if (tc::get_encode() == nullptr) return false;
    return true;
}

static thread_local int g_gemm_mode = MLE_GEMM_MODE_TF32;
// whether large plain products may run on CTA pairs (256-row tiles)
static thread_local int g_gemm_pairs = 1;
// how assigned (not accumulated) outputs leave the epilogue: 0 bulk tensor
// stores, 1 the epilogue warps' own 16-byte stores
static thread_local int g_store_path = 1;
// tile width, split count and pair flag of this thread's last tensor-core launch
static thread_local int g_last_choice[3] = {0, 0, 0};
// Element type of the operand tensor maps: 0 fp32 (the MMA reads the TF32
// part of each value: the low 13 mantissa bits are dropped, a truncation),
// 1 TF32 (the copy engine rounds each fp32 value to the nearest TF32, ties
// to even, as it loads; measured on B200).  Rounding halves the typical
// product error at no cost, so it is the default.
static thread_local int g_operand_round = 1;
static thread_local int g_fuse_colsum = 1;  // column sums beside a product taken in its epilogue warps
static thread_local int g_last_colsum = 0;  // the last product took its column sums so

// k-blocks per stage for products whose operands all have a split view
// (1 forces one k-block per stage everywhere)
static thread_local int g_stage_kblocks = 2;
static thread_local int g_last_kpl = 1;
// forced (tile width, split-K count, CTA pair) for plain products; width 0:
// the tile model decides
static thread_local int g_force_tiles[3] = {0, 0, 0};

// (after the tile model; split-K only where every problem may split, never
// for split-column outputs)
static bool may_split_all(const GemmProblem* ps, int n);
static void apply_forced_tiles(const GemmProblem* ps, int n, int& BN, int& splits, bool& pair) {
    if (g_force_tiles[0] == 0) return;
    for (int i = 0; i < n; ++i)
        if (ps[i].c_split) return;
    BN = g_force_tiles[0];
    splits = may_split_all(ps, n) ? g_force_tiles[1] : 1;
    pair = g_force_tiles[2] != 0;
}

static CUtensorMapDataType operand_type() {
    return g_operand_round ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

namespace {

struct Shape {
    bool A_MN, B_MN;
    int m_tiles, kb_total;
    int64_t z;
};

Shape shape_of(const GemmProblem& p) {
    Shape s;
    s.A_MN = p.trans_a != 0;  // A stored [K][M]: M contiguous
    s.B_MN = p.trans_b == 0;  // B stored [K][N]: N contiguous
    s.z = (int64_t)p.nbatch * p.channels;
    s.m_tiles = (p.M + tc::BM - 1) / tc::BM;
    s.kb_total = (p.K + tc::BK - 1) / tc::BK;
    return s;
}

bool may_split(const GemmProblem& p) {
    const int64_t z = (int64_t)p.nbatch * p.channels;
    const bool c_dense = p.ldc == p.N && (z == 1 || (p.c_sb == (int64_t)p.M * p.N && p.channels == 1));
    return p.mode != tc::EPI_ASSIGN || c_dense;
}

// Tile width and split-K for a set of problems launched together.  For
// accumulated outputs, a fill-time model: operand tiles reach shared memory
// at ~90 GB/s per SM, so the mainloop costs sum M*N*K*4*(1/BN + 1/BM) bytes
// spread over the SMs in use, and splitting K adds one reduce-add of C per
// split.  Its choices match the best measured (BN, splits) within ~5 % for
// the transformer's backward GEMMs.
void choose_tiles(const GemmProblem* ps, int n, int& BN, int& splits, bool model_assign = false,
                  bool* pair = nullptr, bool only_pairs = false) {
    using namespace tc;
    BN = 64;
    splits = 1;
    if (pair) *pair = false;
    // Assigned outputs never split (the memset and reduce-adds cost more
    // than they save, measured on B200); narrow tiles keep enough of them
    // in flight for these small-K products.  `model_assign`: pick the width
    // of an assigned (long-K) product with the fill model instead, as for
    // products of at least two waves of 128 x 128 tiles when CTA pairs are
    // allowed (`pair` non-null).
    bool any_assign = false;
    int max_n = 0;
    int64_t tiles128 = 0;
    double flops = 0;
    for (int i = 0; i < n; ++i) {
        any_assign = any_assign || ps[i].mode == EPI_ASSIGN;
        max_n = std::max(max_n, ps[i].N);
        const Shape sh = shape_of(ps[i]);
        tiles128 += (int64_t)sh.m_tiles * ((ps[i].N + 127) / 128) * sh.z;
        flops += 2.0 * ps[i].M * (double)ps[i].N * ps[i].K * sh.z;
    }
    // pairs only pay with at least a wave of 128 x 128 tiles or a long
    // split-K product (measured on B200: 1024^3 ran slower on pairs, 2048^3
    // and up, and 4096 x 4096 x 256 split over K, faster)
    if (tiles128 < kSMs && flops < 4e9 && !only_pairs) pair = nullptr;
    if (pair && (tiles128 >= 2 * kSMs || only_pairs)) model_assign = true;
    if (any_assign && !model_assign) {
        BN = max_n <= 256 ? 64 : 128;
        return;
    }
    double best = 1e30;
    int min_n = ps[0].N, kb_min = 1 << 30;
    bool split_ok = true;
    for (int i = 0; i < n; ++i) {
        min_n = std::min(min_n, ps[i].N);
        kb_min = std::min(kb_min, shape_of(ps[i]).kb_total);
        split_ok = split_ok && may_split(ps[i]);
    }
    // Model: operand tiles reach shared memory at ~90 GB/s per SM and the
    // tensor pipe retires ~5.5 TFLOP/s per SM (TF32); a CTA pair stages
    // half of its 256 x BN tile's B per SM, so it fills less per FLOP.
    struct Cand {
        int bn;
        bool pr;
    };
    const Cand cands[] = {{256, false}, {128, false}, {64, false}, {256, true}, {128, true}, {64, true}};
    for (const Cand& c : cands) {
        if (c.pr && !pair) continue;
        if (only_pairs && pair && !c.pr) continue;
        const int cand = c.bn, bmt = c.pr ? 2 * BM : BM, per_unit = c.pr ? 2 : 1;
        if (cand > 64 && min_n < cand / 2 + 1) continue;
        int64_t units = 0;
        double fill = 0, flops = 0, cbytes = 0, assign_bytes = 0;
        for (int i = 0; i < n; ++i) {
            const GemmProblem& p = ps[i];
            const Shape sh = shape_of(p);
            const int64_t mt = (p.M + bmt - 1) / bmt;
            const int64_t u = mt * ((p.N + cand - 1) / cand) * sh.z;
            units += u;
            fill += (double)u * (bmt + cand) * (double)sh.kb_total * BK * 4.0;
            flops += 2.0 * (double)u * bmt * cand * (double)sh.kb_total * BK;
            cbytes += (double)p.M * p.N * sh.z * 4.0;
            if (p.mode == EPI_ASSIGN) assign_bytes += (double)p.M * p.N * sh.z * 4.0;
        }
        const int max_split = (split_ok && !any_assign) ? std::max(1, kb_min / 4) : 1;
        const int64_t slots = kSMs / per_unit;
        for (int sp = 1; sp <= max_split; sp = (sp < 4 ? sp + 1 : sp * 2)) {
            const int64_t work = units * sp;
            const double active = (double)std::min<int64_t>(work * per_unit, kSMs);
            double t = std::max(fill / (active * 90e9), flops / (active * 5.5e12)) +
                       0.3e-6 * (double)((work + slots - 1) / slots);
            if (sp > 1) t += (double)sp * cbytes / 3e12 + assign_bytes / 5e12;
            if (t < best * 0.98) {
                best = t;
                BN = cand;
                splits = sp;
                if (pair) *pair = c.pr;
            }
            if (work >= slots) break;
        }
    }
}

// Fills slot g of a launch group for problem p (tensor maps and epilogue
// parameters); an assigned C that is split is zeroed first.  False if TMA
// cannot describe an operand.
int prepare(const GemmProblem& p, int BN, int splits_req, bool force_atomic, tc::GemmGroup& grp, int g,
            cudaStream_t st, bool& ok, bool pair = false, int kpl = 1) {
    using namespace tc;
    ok = false;
    const Shape sh = shape_of(p);
    const int n_tiles = (p.N + BN - 1) / BN;
    const int m_tiles = pair ? (p.M + 2 * BM - 1) / (2 * BM) : sh.m_tiles;  // a pair's tile has 256 rows
    const int bn_cta = pair ? BN / 2 : BN;                                   // B columns a CTA stages
    const int64_t tiles = (int64_t)m_tiles * n_tiles * sh.z;
    const int kb_per_split = (sh.kb_total + splits_req - 1) / splits_req;
    const int splits = (sh.kb_total + kb_per_split - 1) / kb_per_split;
    EpiParams& ep = grp.ep[g];
    memset(&ep, 0, sizeof(ep));
    ep.C = p.C;
    ep.bias = p.bias;
    ep.ldc = p.ldc;
    ep.c_stride_b = p.nbatch == 1 ? 0 : p.c_sb;
    ep.c_stride_c = p.channels == 1 ? 0 : p.c_sc;
    ep.M = p.M;
    ep.N = p.N;
    ep.K = p.K;
    ep.channels = p.channels;
    ep.splits = splits;
    ep.kb_per_split = kb_per_split;
    ep.a_has_b = (p.a_sb != 0 && p.nbatch > 1);
    ep.a_has_c = (p.a_sc != 0 && p.channels > 1);
    ep.b_has_b = (p.b_sb != 0 && p.nbatch > 1);
    ep.b_has_c = (p.b_sc != 0 && p.channels > 1);
    ep.m_tiles = m_tiles;
    ep.n_tiles = n_tiles;
    ep.tiles = tiles * splits;
    ep.alpha = p.alpha;
    ep.mode = (splits > 1 || force_atomic) ? EPI_ATOMIC : p.mode;
    ep.vec = ((p.ldc & 3) == 0) && aligned16(p.C) && ((ep.c_stride_b & 3) == 0) && ((ep.c_stride_c & 3) == 0) &&
             (p.bias == nullptr || aligned16(p.bias));

    OperandView va, vb;
    va.base = p.A;
    va.inner = sh.A_MN ? p.M : p.K;
    va.outer = sh.A_MN ? p.K : p.M;
    va.ld = p.lda;
    va.nc = ep.a_has_c ? p.channels : 1;
    va.nb = ep.a_has_b ? p.nbatch : 1;
    va.sc = p.a_sc;
    va.sb = p.a_sb;
    vb.base = p.B;
    vb.inner = sh.B_MN ? p.N : p.K;
    vb.outer = sh.B_MN ? p.K : p.N;
    vb.ld = p.ldb;
    vb.nc = ep.b_has_c ? p.channels : 1;
    vb.nb = ep.b_has_b ? p.nbatch : 1;
    vb.sc = p.b_sc;
    vb.sb = p.b_sb;
    memset(&grp.a[g], 0, sizeof(CUtensorMap));
    memset(&grp.b[g], 0, sizeof(CUtensorMap));
    memset(&grp.c[g], 0, sizeof(CUtensorMap));
    // split views: always for MN-major operands that have one (one copy
    // instead of one per 32 columns), for K-major ones when the stage holds
    // several k-blocks (kpl > 1 needs both operands split)
    ep.a_split = ((sh.A_MN || kpl > 1) && encode_operand_split(&grp.a[g], va, sh.A_MN, BM, kpl, operand_type())) ? 1 : 0;
    ep.b_split =
        ((sh.B_MN || kpl > 1) && encode_operand_split(&grp.b[g], vb, sh.B_MN, bn_cta, kpl, operand_type())) ? 1 : 0;
    if (kpl > 1 && !(ep.a_split && ep.b_split)) return MLE_OK;
    if (!ep.a_split && !encode_operand(&grp.a[g], va, 32, sh.A_MN ? BK : BM, sh.A_MN, operand_type())) return MLE_OK;
    if (!ep.b_split && !encode_operand(&grp.b[g], vb, 32, sh.B_MN ? BK : bn_cta, sh.B_MN, operand_type()))
        return MLE_OK;
    // C through bulk tensor stores when its rows and strides allow TMA
    ep.c_has_b = (ep.c_stride_b != 0);
    ep.c_has_c = (ep.c_stride_c != 0);
    ep.tma_epi = 0;
    if (p.c_split) {
        // 5-D map (n % c_split, n / c_split, m, channel, batch); only through TMA
        if (p.c_split % 32 || p.N % p.c_split || !aligned16(p.C) || (p.ldc & 3) || (p.c_split_ld & 3) ||
            (ep.c_stride_b & 3) || (ep.c_stride_c & 3) || (splits > 1 && p.mode == EPI_ASSIGN))
            return MLE_OK;
        const int64_t nc = ep.c_has_c ? p.channels : 1, nb = ep.c_has_b ? p.nbatch : 1;
        const int64_t sc = ep.c_has_c ? ep.c_stride_c : (int64_t)p.ldc * p.M;
        const int64_t sb = ep.c_has_b ? ep.c_stride_b : sc * nc;
        const int64_t dims[5] = {p.c_split, p.N / p.c_split, p.M, nc, nb};
        const int64_t str[4] = {p.c_split_ld, p.ldc, sc, sb};
        const int box[5] = {32, 1, 32, 1, 1};
        if (!encode_map(&grp.c[g], p.C, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, 5)) return MLE_OK;
        ep.tma_epi = 1;
        ep.c_split = p.c_split;
        ok = true;
        return MLE_OK;
    }
    const bool assign_out = p.mode == EPI_ASSIGN && splits == 1 && !force_atomic;
    if (aligned16(p.C) && (p.ldc & 3) == 0 && (ep.c_stride_b & 3) == 0 && (ep.c_stride_c & 3) == 0 &&
        !(assign_out && g_store_path == 1)) {
        OperandView vc;
        vc.base = p.C;
        vc.inner = p.N;
        vc.outer = p.M;
        vc.ld = p.ldc;
        vc.nc = ep.c_has_c ? p.channels : 1;
        vc.nb = ep.c_has_b ? p.nbatch : 1;
        vc.sc = ep.c_stride_c;
        vc.sb = ep.c_stride_b;
        ep.tma_epi = encode_operand(&grp.c[g], vc, 32, 32) ? 1 : 0;
    }
    if (splits > 1 && p.mode == EPI_ASSIGN) {
        // split partial products are reduce-added into a zeroed C
        const size_t bytes = sizeof(float) * (size_t)p.M * p.N * (size_t)sh.z;
        if (cudaMemsetAsync(p.C, 0, bytes, st) != cudaSuccess) return launch_status();
    }
    ok = true;
    return MLE_OK;
}

int dispatch(const tc::GemmGroup& grp, bool A_MN, bool B_MN, int BN, cudaStream_t st, bool pair = false,
             int kpl = 1) {
    using namespace tc;
    if (kpl == 2) {  // two k-blocks per stage: half as many stages in the same ring
#define MLE_TCK(AM, BMN, BNV, ST, PR) return launch_tc<AM, BMN, BNV, ST, PR, 2>(grp, st)
#define MLE_TCK4(BNV, ST, PR)                                                        \
    if (A_MN) { if (B_MN) MLE_TCK(true, true, BNV, ST, PR); else MLE_TCK(true, false, BNV, ST, PR); } \
    else { if (B_MN) MLE_TCK(false, true, BNV, ST, PR); else MLE_TCK(false, false, BNV, ST, PR); }
        if (pair) {
            if (BN == 256) { MLE_TCK4(256, 3, true) }
            else if (BN == 128) { MLE_TCK4(128, 4, true) }
            else { MLE_TCK4(64, 4, true) }
        }
        if (BN == 256) { MLE_TCK4(256, 2, false) }
        else if (BN == 128) { MLE_TCK4(128, 3, false) }
        else { MLE_TCK4(64, 4, false) }
#undef MLE_TCK4
#undef MLE_TCK
    }
#define MLE_TC(AM, BMN, BNV, ST) return launch_tc<AM, BMN, BNV, ST>(grp, st)
#define MLE_TC2(AM, BMN, BNV, ST) return launch_tc<AM, BMN, BNV, ST, true>(grp, st)
    if (pair) {  // 256 x BN tiles on CTA pairs, each CTA staging BN/2 columns of B
        if (BN == 256) {
            if (A_MN) { if (B_MN) MLE_TC2(true, true, 256, 6); else MLE_TC2(true, false, 256, 6); }
            else { if (B_MN) MLE_TC2(false, true, 256, 6); else MLE_TC2(false, false, 256, 6); }
        } else if (BN == 128) {
            if (A_MN) { if (B_MN) MLE_TC2(true, true, 128, 7); else MLE_TC2(true, false, 128, 7); }
            else { if (B_MN) MLE_TC2(false, true, 128, 7); else MLE_TC2(false, false, 128, 7); }
        } else {
            if (A_MN) { if (B_MN) MLE_TC2(true, true, 64, 8); else MLE_TC2(true, false, 64, 8); }
            else { if (B_MN) MLE_TC2(false, true, 64, 8); else MLE_TC2(false, false, 64, 8); }
        }
    }
#undef MLE_TC2
    if (BN == 256) {
        if (A_MN) { if (B_MN) MLE_TC(true, true, 256, 4); else MLE_TC(true, false, 256, 4); }
        else { if (B_MN) MLE_TC(false, true, 256, 4); else MLE_TC(false, false, 256, 4); }
    } else if (BN == 128) {
        if (A_MN) { if (B_MN) MLE_TC(true, true, 128, 5); else MLE_TC(true, false, 128, 5); }
        else { if (B_MN) MLE_TC(false, true, 128, 5); else MLE_TC(false, false, 128, 5); }
    } else {
        if (A_MN) { if (B_MN) MLE_TC(true, true, 64, 6); else MLE_TC(true, false, 64, 6); }
        else { if (B_MN) MLE_TC(false, true, 64, 6); else MLE_TC(false, false, 64, 6); }
    }
#undef MLE_TC
}

bool tc_path(const GemmProblem& p) { return p.K > 0 && g_gemm_mode == MLE_GEMM_MODE_TF32 && tc_eligible(p); }

}  // namespace

static bool may_split_all(const GemmProblem* ps, int n) {
    for (int i = 0; i < n; ++i)
        if (!may_split(ps[i])) return false;
    return true;
}

namespace {

// Both operands have a split view (contiguous extent a multiple of 32):
// the product may stage two k-blocks per copy.
bool split_ok(const GemmProblem& p) {
    const Shape sh = shape_of(p);
    return (sh.A_MN ? p.M % 32 == 0 : p.K % 32 == 0) && (sh.B_MN ? p.N % 32 == 0 : p.K % 32 == 0);
}

}  // namespace

namespace {

template <int MODE, int HD, int SQ>
int launch_attn_keys(const tc::AttnKeysParams& prm, int64_t ctas, cudaStream_t st) {
    using L = tc::AttnKeysSmem<HD, SQ>;
    static_assert(2 * L::TOTAL <= 228 * 1024 || HD > 64, "two CTAs per SM");
    auto kern = tc::attn_keys_kernel<MODE, HD, SQ>;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) != cudaSuccess)
            return launch_status();
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(128 * tc::attn_keys_groups<MODE>());
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, prm) != cudaSuccess) return launch_status();
    return launch_status();
}

}  // namespace

bool attn_keys_supported(int Sq, int Sk, int hd, int64_t BH) {
    return Sq > 0 && Sq <= 256 && Sk > 0 && (hd == 32 || hd == 64 || hd == 128) &&
           BH * ((Sk + 127) / 128) <= 0x7fffffff && tc::get_encode() != nullptr;
}

int run_attn_keys(int mode, const float* keys_src, const float* rows_src, const float* P, float* out, int B, int H,
                  int Sq, int Sk, int hd, int64_t key_b, int64_t key_h, int64_t key_s, int64_t row_b, int64_t row_h,
                  int64_t row_s, float scale, int causal, cudaStream_t st, float* stats) {
    if (!attn_keys_supported(Sq, Sk, hd, (int64_t)B * H)) return MLE_ERR_UNSUPPORTED;
    if (mode == 0 && !out && !stats) return MLE_ERR_ARG;
    tc::AttnKeysParams prm;
    memset(&prm, 0, sizeof(prm));
    const int SQ = Sq <= 128 ? 128 : 256;
    const int64_t kd[4] = {hd, Sk, H, B}, ks[3] = {key_s, key_h, key_b};
    const int64_t rd[4] = {hd, Sq, H, B}, rs[3] = {row_s, row_h, row_b};
    const int kbox[4] = {32, 128, 1, 1}, rbox[4] = {32, SQ, 1, 1};
    if (!tc::encode_map(&prm.a_map, keys_src, kd, ks, kbox, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()) ||
        !tc::encode_map(&prm.b_map, rows_src, rd, rs, rbox, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()))
        return MLE_ERR_UNSUPPORTED;
    prm.P = P;
    prm.out = out;
    prm.stats = mode == 0 ? stats : nullptr;
    prm.H = H;
    prm.Sq = Sq;
    prm.Sk = Sk;
    prm.key_blocks = (Sk + 127) / 128;
    prm.scale = scale;
    prm.causal = causal;
    const int64_t ctas = (int64_t)B * H * prm.key_blocks;
    auto go = [&](auto m, auto d, auto q) {
        return launch_attn_keys<decltype(m)::value, decltype(d)::value, decltype(q)::value>(prm, ctas, st);
    };
    using std::integral_constant;
#define MLE_AK(MO, HDV)                                                                                     \
    if (mode == MO && hd == HDV)                                                                            \
        return SQ == 128 ? go(integral_constant<int, MO>(), integral_constant<int, HDV>(), integral_constant<int, 128>()) \
                         : go(integral_constant<int, MO>(), integral_constant<int, HDV>(), integral_constant<int, 256>());
    MLE_AK(0, 32)
    MLE_AK(0, 64)
    MLE_AK(0, 128)
    MLE_AK(1, 32)
    MLE_AK(1, 64)
    MLE_AK(1, 128)
#undef MLE_AK
    return MLE_ERR_UNSUPPORTED;
}

#include "attention_flash.cuh"

// Column sums of B requested beside a product (GemmProblem::colsum): those
// the launch takes in its epilogue warps are attached to the group; the rest
// follow as column-sum launches (finish_colsums).
static bool colsum_fusable(const GemmProblem& p, bool) {
    return g_fuse_colsum && p.colsum && !p.trans_b && p.nbatch == 1 && p.channels == 1 && p.ldb == p.N;
}

static int column_sums(const GemmProblem& p, cudaStream_t st) {
    if (!p.colsum || p.K <= 0) return MLE_OK;
    if (p.trans_b || p.ldb != p.N || p.nbatch != 1 || p.channels != 1) return MLE_ERR_UNSUPPORTED;
    return mle_bias_grad(p.B, p.colsum, p.K, p.N, 1.0f, reinterpret_cast<mle_stream_t>(st));
}

static void attach_colsums(const GemmProblem* ps, int n, tc::GemmGroup& grp, bool pair, bool* post) {
    // Once a launch sums columns its epilogue warps release every stage, so
    // a CTA with several tiles no longer overlaps one tile's epilogue with
    // the next tile's mainloop (8192^3: +0.7 ms against +0.3 ms for the
    // separate sum): fused only where every CTA has at most one tile.
    int64_t tiles = 0;
    for (int i = 0; i < (grp.n > 1 ? grp.n : 1); ++i) tiles += grp.ep[i].tiles;
    const bool one_wave = tiles * (pair ? 2 : 1) <= (int64_t)kSMs;
    g_last_colsum = 0;
    for (int i = 0; i < n; ++i) {
        post[i] = false;
        if (!ps[i].colsum) continue;
        if (one_wave && colsum_fusable(ps[i], pair) && grp.kcat <= 1 && grp.ep[i].conv == 0) {
            grp.ep[i].colsum = ps[i].colsum;
            grp.colsum = 1;
            g_last_colsum = 1;
        } else {
            post[i] = true;
        }
    }
}

static int finish_colsums(const GemmProblem* ps, int n, const bool* post, cudaStream_t st) {
    for (int i = 0; i < n; ++i)
        if (post[i]) {
            const int s = column_sums(ps[i], st);
            if (s) return s;
        }
    return MLE_OK;
}

int run_gemm(const GemmProblem& p, cudaStream_t st) {
    if (p.M <= 0 || p.N <= 0 || p.nbatch <= 0 || p.channels <= 0) return MLE_OK;
    if (p.colsum && (p.trans_b || p.ldb != p.N || p.nbatch != 1 || p.channels != 1)) return MLE_ERR_UNSUPPORTED;
    if (p.K <= 0) {
        // empty reduction: assign writes alpha*0 (+bias); accumulate is a no-op
        if (p.mode != tc::EPI_ASSIGN) return MLE_OK;
    }
    if (!tc_path(p)) {
        if (p.c_split) return MLE_ERR_UNSUPPORTED;
        const int s = simt_gemm(p, st);
        return s ? s : column_sums(p, st);
    }
    int BN, splits;
    bool pair = false;
    choose_tiles(&p, 1, BN, splits, false, g_gemm_pairs ? &pair : nullptr, g_gemm_pairs == 2);
    apply_forced_tiles(&p, 1, BN, splits, pair);
    tc::GemmGroup grp;
    memset(&grp, 0, sizeof(grp));
    bool ok = false;
    int kpl = (g_stage_kblocks == 2 && split_ok(p)) ? 2 : 1;
    int s = prepare(p, BN, splits, false, grp, 0, st, ok, pair, kpl);
    if (s) return s;
    if (!ok && kpl == 2) {
        kpl = 1;
        memset(&grp, 0, sizeof(grp));
        s = prepare(p, BN, splits, false, grp, 0, st, ok, pair, kpl);
        if (s) return s;
    }
    if (!ok) {
        if (p.c_split) return MLE_ERR_UNSUPPORTED;
        const int s2 = simt_gemm(p, st);
        return s2 ? s2 : column_sums(p, st);
    }
    grp.n = 1;
    grp.tile_start[0] = 0;
    grp.tile_start[1] = grp.ep[0].tiles;
    const Shape sh = shape_of(p);
    g_last_choice[0] = BN;
    g_last_choice[1] = grp.ep[0].splits;
    g_last_choice[2] = pair ? 1 : 0;
    g_last_kpl = kpl;
    bool post[1];
    attach_colsums(&p, 1, grp, pair, post);
    s = dispatch(grp, sh.A_MN, sh.B_MN, BN, st, pair, kpl);
    return s ? s : finish_colsums(&p, 1, post, st);
}

// Problems of one layout class in one persistent launch.  `shared_c`: all
// write the same C (their results are summed with reduce-adds).  Falls back
// to one launch per problem when the set cannot share a launch.
int run_gemm_group(const GemmProblem* ps, int n, bool shared_c, cudaStream_t st) {
    if (n <= 0) return MLE_OK;
    bool same = n <= tc::kMaxGroup;
    for (int i = 0; i < n && same; ++i) {
        same = tc_path(ps[i]) && ps[i].M > 0 && ps[i].N > 0 && ps[i].nbatch > 0 && ps[i].channels > 0 &&
               shape_of(ps[i]).A_MN == shape_of(ps[0]).A_MN && shape_of(ps[i]).B_MN == shape_of(ps[0]).B_MN;
        if (shared_c && ps[i].mode == tc::EPI_ASSIGN) same = false;
    }
    if (!same) {
        for (int i = 0; i < n; ++i) {
            const int s = run_gemm(ps[i], st);
            if (s) return s;
        }
        return MLE_OK;
    }
    int BN, splits;
    bool pair = false;
    choose_tiles(ps, n, BN, splits, false, g_gemm_pairs ? &pair : nullptr, g_gemm_pairs == 2);
    apply_forced_tiles(ps, n, BN, splits, pair);
    tc::GemmGroup grp;
    int kpl = g_stage_kblocks == 2 ? 2 : 1;
    for (int i = 0; i < n; ++i) kpl = split_ok(ps[i]) ? kpl : 1;
    for (;;) {
        memset(&grp, 0, sizeof(grp));
        grp.n = n;
        grp.tile_start[0] = 0;
        bool all_ok = true;
        for (int i = 0; i < n && all_ok; ++i) {
            bool ok = false;
            const int s = prepare(ps[i], BN, splits, shared_c, grp, i, st, ok, pair, kpl);
            if (s) return s;
            all_ok = ok;
            grp.tile_start[i + 1] = grp.tile_start[i] + grp.ep[i].tiles;
        }
        if (all_ok) break;
        if (kpl == 2) {  // a split view TMA cannot describe: one k-block per stage
            kpl = 1;
            continue;
        }
        // an operand TMA cannot describe: separate launches
        for (int j = 0; j < n; ++j) {
            const int s2 = run_gemm(ps[j], st);
            if (s2) return s2;
        }
        return MLE_OK;
    }
    // problems reading the same A over the same tile rows walk them together
    bool ilv = n > 1;
    for (int i = 1; i < n && ilv; ++i)
        ilv = ps[i].A == ps[0].A && ps[i].lda == ps[0].lda && grp.ep[i].m_tiles == grp.ep[0].m_tiles &&
              grp.ep[i].splits == grp.ep[0].splits && grp.ep[i].kb_per_split == grp.ep[0].kb_per_split &&
              ps[i].nbatch == ps[0].nbatch && ps[i].channels == ps[0].channels;
    if (ilv) {
        grp.ilv = 1;
        grp.ilv_n[0] = 0;
        for (int i = 0; i < n; ++i) grp.ilv_n[i + 1] = grp.ilv_n[i] + grp.ep[i].n_tiles;
    }
    g_last_kpl = kpl;
    bool post[tc::kMaxGroup];
    attach_colsums(ps, n, grp, pair, post);
    const int s = dispatch(grp, shape_of(ps[0]).A_MN, shape_of(ps[0]).B_MN, BN, st, pair, kpl);
    return s ? s : finish_colsums(ps, n, post, st);
}

int run_gemm_kcat(const GemmProblem* ps, int n, cudaStream_t st) {
    using namespace tc;
    if (n <= 1) return n == 1 ? run_gemm(ps[0], st) : MLE_OK;
    // one output, one launch, each A_g B_g product a segment of the
    // reduction: C, M, N, layouts, mode and alpha shared, unbatched
    bool ok = n <= kMaxGroup;
    int64_t ksum = 0;
    for (int i = 0; i < n && ok; ++i) {
        const GemmProblem& p = ps[i];
        ok = tc_path(p) && p.C == ps[0].C && p.M == ps[0].M && p.N == ps[0].N && p.ldc == ps[0].ldc &&
             p.mode == ps[0].mode && p.alpha == ps[0].alpha && p.nbatch == 1 && p.channels == 1 && !p.bias &&
             !p.c_split && !p.colsum && p.mode != EPI_ATOMIC && p.K > 0 && p.K % 64 == 0 &&
             shape_of(p).A_MN == shape_of(ps[0]).A_MN && shape_of(p).B_MN == shape_of(ps[0]).B_MN;
        ksum += p.K;
    }
    if (!ok || ksum > 0x7fffffff) return run_gemm_group(ps, n, true, st);
    GemmProblem whole = ps[0];
    whole.K = (int)ksum;
    int BN, splits;
    bool pair = false;
    choose_tiles(&whole, 1, BN, splits, false, g_gemm_pairs ? &pair : nullptr, g_gemm_pairs == 2);
    apply_forced_tiles(&whole, 1, BN, splits, pair);
    int kpl = g_stage_kblocks == 2 ? 2 : 1;
    for (int i = 0; i < n; ++i) kpl = split_ok(ps[i]) ? kpl : 1;
    tc::GemmGroup grp;
    for (;;) {
        memset(&grp, 0, sizeof(grp));
        bool all_ok = true;
        // every segment's operand maps; the tile walk and epilogue are ep[0]'s
        for (int i = 0; i < n && all_ok; ++i) {
            bool seg_ok = false;
            const int s = prepare(ps[i], BN, 1, false, grp, i, st, seg_ok, pair, kpl);
            if (s) return s;
            all_ok = seg_ok;
        }
        if (all_ok) break;
        if (kpl == 2) {
            kpl = 1;
            continue;
        }
        return run_gemm_group(ps, n, true, st);
    }
    grp.n = 1;
    grp.kcat = n;
    grp.kcat_kb[0] = 0;
    for (int i = 0; i < n; ++i) grp.kcat_kb[i + 1] = grp.kcat_kb[i] + ps[i].K / BK;
    grp.ep[0].K = (int)ksum;
    grp.ep[0].splits = 1;
    grp.ep[0].kb_per_split = grp.kcat_kb[n];
    grp.tile_start[0] = 0;
    grp.tile_start[1] = grp.ep[0].tiles;
    g_last_kpl = kpl;
    return dispatch(grp, shape_of(ps[0]).A_MN, shape_of(ps[0]).B_MN, BN, st, pair, kpl);
}

bool conv_gemm_supported(const ConvGemm& c) {
    if (g_gemm_mode != MLE_GEMM_MODE_TF32 || tc::get_encode() == nullptr) return false;
    if (c.kind != 1 && c.kind != 2) return false;
    if (c.M <= 0 || c.C <= 0 || c.HS <= 0 || c.WS <= 0 || c.KH <= 0 || c.KW <= 0 || c.nb <= 0 || c.P <= 0)
        return false;
    // a tap moves the flattened pixel index by whole rows, which keeps TMA
    // x coordinates at multiples of 4 elements (16 bytes)
    if (c.WS & 3) return false;
    if ((c.P & 3) || !aligned16(c.A) || !aligned16(c.S) || !aligned16(c.out)) return false;
    if (c.kind == 1 && ((c.lda & 3) || c.lda < c.C)) return false;
    if (c.kind == 2 && ((c.ldc & 3) || c.ldc < c.C)) return false;
    return true;
}

// Kind 1 with output pixels as the tile rows (EpiParams::conv == 3): the
// output channels become the tile columns, so a narrow channel count (64)
// fills a 64-wide tile instead of half of a 128-row one, and the bias is
// added in the epilogue.  Returns false (nothing launched) when TMA cannot
// describe the transposed output.
static bool run_conv_gemm_swapped(const ConvGemm& c, cudaStream_t st, int& status) {
    using namespace tc;
    const int taps = c.KH * c.KW;
    const int cblk = (c.C + BK - 1) / BK;
    GemmProblem q;
    memset(&q, 0, sizeof(q));
    q.M = c.P;
    q.N = c.M;
    q.K = taps * cblk * BK;
    q.nbatch = c.nb;
    q.channels = 1;
    q.ldc = c.P;
    q.alpha = 1.f;
    q.mode = c.accumulate ? EPI_ACCUM : EPI_ASSIGN;
    int BN, splits;
    bool pair = false;
    choose_tiles(&q, 1, BN, splits, true, g_gemm_pairs ? &pair : nullptr, g_gemm_pairs == 2);
    const int kb_total = taps * cblk;
    const int kb_per_split = (kb_total + splits - 1) / splits;
    splits = (kb_total + kb_per_split - 1) / kb_per_split;
    GemmGroup grp;
    memset(&grp, 0, sizeof(grp));
    EpiParams& ep = grp.ep[0];
    ep.C = c.out;
    ep.bias = c.bias;
    ep.alpha = 1.f;
    ep.M = c.P;
    ep.N = c.M;
    ep.K = q.K;
    ep.ldc = c.P;
    ep.c_stride_b = c.nb > 1 ? (int64_t)c.M * c.P : 0;
    ep.channels = 1;
    ep.splits = splits;
    ep.kb_per_split = kb_per_split;
    ep.m_tiles = (c.P + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
    ep.n_tiles = (c.M + BN - 1) / BN;
    ep.mode = splits > 1 ? EPI_ATOMIC : (c.accumulate ? EPI_ACCUM : EPI_ASSIGN);
    ep.conv = 3;
    ep.cv_kw = c.KW;
    ep.cv_pad = c.pad;
    ep.cv_w = c.WS;
    ep.cv_nb = c.nb;
    ep.cv_cblk = cblk;
    ep.c_trans = 1;
    ep.c_has_b = c.nb > 1;
    ep.vec = aligned16(c.out) && (c.bias == nullptr || aligned16(c.bias));
    const int64_t plane = (int64_t)c.HS * c.WS;
    const int64_t s_dims[4] = {plane, c.C, (int64_t)c.KW * c.nb, 1};
    const int64_t s_str[3] = {plane, plane * c.C, plane * c.C * c.KW * c.nb};
    const int s_box[4] = {32, BK, 1, 1};
    const int64_t w_dims[4] = {c.lda, c.M, taps, 1};
    const int64_t w_str[3] = {c.lda, (int64_t)c.M * c.lda, (int64_t)taps * c.M * c.lda};
    const int w_box[4] = {BK, pair ? BN / 2 : BN, 1, 1};
    const int64_t c_dims[4] = {c.P, c.M, 1, c.nb};
    const int64_t c_str[3] = {c.P, (int64_t)c.M * c.P, (int64_t)c.M * c.P};
    const int c_box[4] = {32, 32, 1, 1};
    if (!encode_map(&grp.a[0], c.S, s_dims, s_str, s_box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, 4, operand_type()) ||
        !encode_map(&grp.b[0], c.A, w_dims, w_str, w_box, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()) ||
        !encode_map(&grp.c[0], c.out, c_dims, c_str, c_box, CU_TENSOR_MAP_SWIZZLE_128B))
        return false;
    ep.tma_epi = 1;
    if (splits > 1 && !c.accumulate) {
        // split partial products are reduce-added into a zeroed output
        if (cudaMemsetAsync(c.out, 0, sizeof(float) * (size_t)c.nb * c.M * c.P, st) != cudaSuccess) {
            status = launch_status();
            return true;
        }
    }
    ep.tiles = (int64_t)ep.m_tiles * ep.n_tiles * c.nb * splits;
    grp.n = 1;
    grp.tile_start[0] = 0;
    grp.tile_start[1] = ep.tiles;
    status = dispatch(grp, true, false, BN, st, pair);
    return true;
}

int run_conv_gemm(const ConvGemm& c, cudaStream_t st) {
    using namespace tc;
    if (!conv_gemm_supported(c)) return MLE_ERR_ARG;
    const int taps = c.KH * c.KW;
    if (c.kind == 1) {
        // pixel rows unless the padded tile area says otherwise
        auto up = [](int64_t v, int64_t m) { return (v + m - 1) / m * m; };
        const int64_t area_n = up(c.M, BM) * up(c.P, 64), area_t = up(c.P, BM) * up(c.M, 64);
        int status = MLE_OK;
        if (area_t <= area_n && run_conv_gemm_swapped(c, st, status)) return status;
    }
    // tile choice on the equivalent plain products
    GemmProblem q;
    memset(&q, 0, sizeof(q));
    q.M = c.M;
    q.channels = 1;
    q.alpha = 1.f;
    if (c.kind == 1) {
        q.N = c.P;
        q.K = taps * ((c.C + BK - 1) / BK) * BK;
        q.nbatch = c.nb;
        q.ldc = c.P;
        q.c_sb = (int64_t)c.M * c.P;
        q.mode = c.accumulate ? EPI_ACCUM : EPI_ASSIGN;
    } else {
        q.N = c.C;
        q.K = c.P;
        q.nbatch = c.nb * taps;
        q.ldc = c.ldc;
        q.mode = EPI_ACCUM;
    }
    int BN, splits;
    bool pair = false;
    choose_tiles(&q, 1, BN, splits, false, g_gemm_pairs ? &pair : nullptr, g_gemm_pairs == 2);
    const int kb_total = (q.K + BK - 1) / BK;
    const int kb_per_split = (kb_total + splits - 1) / splits;
    splits = (kb_total + kb_per_split - 1) / kb_per_split;

    GemmGroup grp;
    memset(&grp, 0, sizeof(grp));
    EpiParams& ep = grp.ep[0];
    ep.C = c.out;
    ep.alpha = 1.f;
    ep.M = c.M;
    ep.K = q.K;
    ep.channels = 1;
    ep.splits = splits;
    ep.kb_per_split = kb_per_split;
    ep.m_tiles = (c.M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
    ep.conv = c.kind;
    ep.cv_kw = c.KW;
    ep.cv_pad = c.pad;
    ep.cv_w = c.WS;
    ep.cv_nb = c.nb;
    // shifted copies as [KW*nb][C][HS*WS]: rows outside the image read as 0
    const int64_t plane = (int64_t)c.HS * c.WS;
    const int64_t s_dims[4] = {plane, c.C, (int64_t)c.KW * c.nb, 1};
    const int64_t s_str[3] = {plane, plane * c.C, plane * c.C * c.KW * c.nb};
    if (c.kind == 1) {
        ep.N = c.P;
        ep.ldc = c.P;
        ep.c_stride_b = c.nb > 1 ? (int64_t)c.M * c.P : 0;
        ep.cv_cblk = (c.C + BK - 1) / BK;
        ep.n_tiles = (c.P + BN - 1) / BN;
        ep.mode = splits > 1 ? EPI_ATOMIC : (c.accumulate ? EPI_ACCUM : EPI_ASSIGN);
        const int64_t a_dims[4] = {c.lda, c.M, taps, 1};
        const int64_t a_str[3] = {c.lda, (int64_t)c.M * c.lda, (int64_t)taps * c.M * c.lda};
        const int a_box[4] = {BK, BM, 1, 1};
        const int s_box[4] = {32, BK, 1, 1};
        if (!encode_map(&grp.a[0], c.A, a_dims, a_str, a_box, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()) ||
            !encode_map(&grp.b[0], c.S, s_dims, s_str, s_box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, 4,
                        operand_type()))
            return MLE_ERR_ARG;
        const int64_t c_dims[4] = {c.P, c.M, 1, c.nb};
        const int64_t c_str[3] = {c.P, (int64_t)c.M * c.P, (int64_t)c.M * c.P};
        const int c_box[4] = {32, 32, 1, 1};
        ep.tma_epi = encode_map(&grp.c[0], c.out, c_dims, c_str, c_box, CU_TENSOR_MAP_SWIZZLE_128B) ? 1 : 0;
        ep.c_has_b = c.nb > 1;
    } else {
        ep.N = c.C;
        ep.ldc = c.ldc;
        ep.c_stride_c = (int64_t)c.M * c.ldc;
        ep.cv_cblk = (c.C + BN - 1) / BN;
        ep.n_tiles = taps * ep.cv_cblk;
        ep.mode = EPI_ATOMIC;
        ep.a_has_b = c.nb > 1;
        const int64_t a_dims[4] = {c.P, c.M, 1, c.nb};
        const int64_t a_str[3] = {c.P, (int64_t)c.M * c.P, (int64_t)c.M * c.P};
        const int a_box[4] = {BK, BM, 1, 1};
        const int s_box[4] = {32, pair ? BN / 2 : BN, 1, 1};
        if (!encode_map(&grp.a[0], c.A, a_dims, a_str, a_box, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()) ||
            !encode_map(&grp.b[0], c.S, s_dims, s_str, s_box, CU_TENSOR_MAP_SWIZZLE_128B, 4, operand_type()))
            return MLE_ERR_ARG;
        const int64_t c_dims[4] = {c.C, c.M, taps, 1};
        const int64_t c_str[3] = {c.ldc, (int64_t)c.M * c.ldc, (int64_t)taps * c.M * c.ldc};
        const int c_box[4] = {32, 32, 1, 1};
        ep.tma_epi = encode_map(&grp.c[0], c.out, c_dims, c_str, c_box, CU_TENSOR_MAP_SWIZZLE_128B) ? 1 : 0;
        ep.c_has_c = 1;
    }
    ep.vec = ((ep.ldc & 3) == 0) && aligned16(c.out);
    ep.tiles = (int64_t)ep.m_tiles * ep.n_tiles * c.nb * splits;
    grp.n = 1;
    grp.tile_start[0] = 0;
    grp.tile_start[1] = ep.tiles;
    if (ep.tiles == 0) return MLE_OK;
    const int s = dispatch(grp, false, c.kind == 1, BN, st, pair);
    if (s || c.kind != 1 || !c.bias) return s;
    // the bias runs along the tile rows here: a separate pass
    return mle_channel_bias_fwd(c.out, c.bias, c.out, c.nb, c.M, c.P, st);
}

}  // namespace mle

using namespace mle;

extern "C" {

int mle_set_gemm_mode(int mode) {
    if (mode != MLE_GEMM_MODE_TF32 && mode != MLE_GEMM_MODE_FP32) return MLE_ERR_ARG;
    g_gemm_mode = mode;
    return MLE_OK;
}

int mle_get_gemm_mode(void) { return g_gemm_mode; }

int mle_set_gemm_pairs(int enable) {
    if (enable < 0 || enable > 2) return MLE_ERR_ARG;
    g_gemm_pairs = enable;
    return MLE_OK;
}

int mle_get_gemm_pairs(void) { return g_gemm_pairs; }

int mle_set_gemm_store_path(int path) {
    if (path != 0 && path != 1) return MLE_ERR_ARG;
    g_store_path = path;
    return MLE_OK;
}

int mle_set_gemm_tiles(int bn, int splits, int pair) {
    if (bn == 0) {
        g_force_tiles[0] = g_force_tiles[1] = g_force_tiles[2] = 0;
        return MLE_OK;
    }
    if ((bn != 64 && bn != 128 && bn != 256) || splits < 1 || splits > 64 || (pair != 0 && pair != 1))
        return MLE_ERR_ARG;
    g_force_tiles[0] = bn;
    g_force_tiles[1] = splits;
    g_force_tiles[2] = pair;
    return MLE_OK;
}

int mle_set_gemm_stage_kblocks(int kblocks) {
    if (kblocks != 1 && kblocks != 2) return MLE_ERR_ARG;
    g_stage_kblocks = kblocks;
    return MLE_OK;
}

int mle_get_gemm_stage_kblocks(void) { return g_stage_kblocks; }

int mle_gemm_last_stage_kblocks(void) { return g_last_kpl; }

int mle_set_gemm_operand_rounding(int mode) {
    if (mode != 0 && mode != 1) return MLE_ERR_ARG;
    g_operand_round = mode;
    return MLE_OK;
}

int mle_get_gemm_operand_rounding(void) { return g_operand_round; }

int mle_set_gemm_column_sums(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    g_fuse_colsum = enable;
    return MLE_OK;
}

int mle_get_gemm_column_sums(void) { return g_fuse_colsum; }

int mle_gemm_last_column_sums(void) { return g_last_colsum; }

int mle_gemm_last_choice(int* out3) {
    if (!out3) return MLE_ERR_ARG;
    for (int i = 0; i < 3; ++i) out3[i] = g_last_choice[i];
    return MLE_OK;
}

int mle_watchdog_read(int* out_flag, mle_stream_t stream) {
    if (!out_flag) return MLE_ERR_ARG;
    unsigned int v = 0, zero = 0;
    cudaStream_t st = as_stream(stream);
    if (cudaMemcpyFromSymbolAsync(&v, g_tc_watchdog, sizeof(v), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return launch_status();
    if (cudaMemcpyToSymbolAsync(g_tc_watchdog, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return launch_status();
    if (cudaStreamSynchronize(st) != cudaSuccess) return launch_status();
    *out_flag = (int)v;
    return MLE_OK;
}

int mle_gemm(const float* A, const float* B, float* C, const float* bias, int batch, int64_t M, int64_t N, int64_t K,
             int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a, int64_t stride_b, int64_t stride_c, int trans_a,
             int trans_b, float alpha, float beta, mle_stream_t stream) {
    if (!A || !B || !C || batch <= 0 || M < 0 || N < 0 || K < 0) return MLE_ERR_ARG;
    if (beta != 0.0f && beta != 1.0f) return MLE_ERR_UNSUPPORTED;
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return MLE_ERR_UNSUPPORTED;
    g_last_kpl = 0;  // set again if the product runs on the tensor cores
    GemmProblem p;
    p.A = A;
    p.B = B;
    p.C = C;
    p.bias = bias;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.lda = lda;
    p.ldb = ldb;
    p.ldc = ldc;
    p.trans_a = trans_a;
    p.trans_b = trans_b;
    p.nbatch = batch;
    p.channels = 1;
    p.a_sb = (batch > 1) ? stride_a : 0;
    p.b_sb = (batch > 1) ? stride_b : 0;
    p.c_sb = (batch > 1) ? stride_c : 0;
    p.a_sc = p.b_sc = p.c_sc = 0;
    p.alpha = alpha;
    p.mode = (beta == 0.0f) ? tc::EPI_ASSIGN : tc::EPI_ACCUM;
    if (batch > 1 && stride_c == 0) {
        if (beta == 0.0f) return MLE_ERR_UNSUPPORTED;
        p.mode = tc::EPI_ATOMIC;
    }
    return run_gemm(p, as_stream(stream));
}

namespace {
// A single (unbatched) row-major product as the Linear entry points use it.
GemmProblem linear_problem(const float* A, const float* B, float* C, const float* bias, int64_t M, int64_t N,
                           int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int trans_a, int trans_b, int mode) {
    GemmProblem p;
    memset(&p, 0, sizeof(p));
    p.A = A;
    p.B = B;
    p.C = C;
    p.bias = bias;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.lda = lda;
    p.ldb = ldb;
    p.ldc = ldc;
    p.trans_a = trans_a;
    p.trans_b = trans_b;
    p.nbatch = 1;
    p.channels = 1;
    p.alpha = 1.0f;
    p.mode = mode;
    return p;
}
}  // namespace

int mle_linear_group_fwd(const float* X, const float* const* W, const float* const* bias, float* const* Y, int n,
                         int64_t rows, int in_features, const int* out_features, mle_stream_t stream) {
    if (!X || !W || !Y || !out_features || n <= 0 || n > tc::kMaxGroup || rows < 0 || in_features <= 0)
        return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    if (rows > 0x7fffffff) return MLE_ERR_UNSUPPORTED;
    GemmProblem ps[tc::kMaxGroup];
    for (int i = 0; i < n; ++i) {
        if (!W[i] || !Y[i] || out_features[i] <= 0) return MLE_ERR_ARG;
        ps[i] = linear_problem(X, W[i], Y[i], bias ? bias[i] : nullptr, rows, out_features[i], in_features,
                               in_features, out_features[i], out_features[i], 0, 0, tc::EPI_ASSIGN);
    }
    return run_gemm_group(ps, n, false, as_stream(stream));
}

int mle_linear_group_bwd(const float* X, const float* const* W, const float* const* dY, float* dX,
                         float* const* dW, float* const* dB, int n, int64_t rows, int in_features,
                         const int* out_features, mle_stream_t stream) {
    if ((dW && !X) || !W || !dY || !out_features || n <= 0 || n > tc::kMaxGroup || rows < 0 || in_features <= 0)
        return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    if (rows > 0x7fffffff) return MLE_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    GemmProblem ps[tc::kMaxGroup];
    int s;
    if (dX) {
        // dX += sum_i dY_i W_i^T: one product over the concatenated
        // reduction (K = sum of out_features), dX read and written once
        for (int i = 0; i < n; ++i) {
            if (!W[i] || !dY[i] || out_features[i] <= 0) return MLE_ERR_ARG;
            ps[i] = linear_problem(dY[i], W[i], dX, nullptr, rows, in_features, out_features[i], out_features[i],
                                   out_features[i], in_features, 0, 1, tc::EPI_ACCUM);
        }
        s = run_gemm_kcat(ps, n, st);
        if (s) return s;
    }
    // dW_i += X^T dY_i
    if (dW) {
        for (int i = 0; i < n; ++i) {
            if (!dW[i] || !dY[i] || out_features[i] <= 0) return MLE_ERR_ARG;
            ps[i] = linear_problem(X, dY[i], dW[i], nullptr, in_features, out_features[i], rows, in_features,
                                   out_features[i], out_features[i], 1, 0, tc::EPI_ACCUM);
            ps[i].colsum = dB ? dB[i] : nullptr;
        }
        return run_gemm_group(ps, n, false, st);
    }
    if (dB) {
        for (int i = 0; i < n; ++i) {
            if (!dB[i]) continue;
            s = mle_bias_grad(dY[i], dB[i], rows, out_features[i], 1.0f, stream);
            if (s) return s;
        }
    }
    return MLE_OK;
}

int mle_bcmm(int variant, const float* A, const float* B, float* C, int batch, int channels, int m, int n, int p,
             int backward, int A_case, int B_case, int C_case, float scale, mle_stream_t stream) {
    if (!A || !B || !C || batch <= 0 || channels <= 0 || m <= 0 || n <= 0 || p <= 0) return MLE_ERR_ARG;
    if (variant < 0 || variant > 3 || A_case < 0 || A_case > 3 || B_case < 0 || B_case > 3 || C_case < 0 ||
        C_case > 3)
        return MLE_ERR_ARG;
    // Per-operand element strides for batch and channel, as batch_chan_offset
    // (Engine/kernels.cu:371-385) computes them.
    auto strides = [&](int flag, int64_t inner, int64_t& sb, int64_t& sc) {
        const int hb = flag & 1, hc = (flag >> 1) & 1;
        sc = hc ? inner : 0;
        sb = hb ? (hc ? (int64_t)channels * inner : inner) : 0;
    };
    const bool a_t = (variant == MLE_GEMM_ATB || variant == MLE_GEMM_ATBT);
    const bool b_t = (variant == MLE_GEMM_ABT || variant == MLE_GEMM_ATBT);
    GemmProblem q;
    q.A = A;
    q.B = B;
    q.C = C;
    q.bias = nullptr;
    q.M = m;
    q.N = p;
    q.K = n;
    q.lda = a_t ? m : n;  // A stored [n][m] when transposed
    q.ldb = b_t ? n : p;  // B stored [p][n] when transposed
    q.ldc = p;
    q.trans_a = a_t;
    q.trans_b = b_t;
    strides(A_case, (int64_t)m * n, q.a_sb, q.a_sc);
    strides(B_case, (int64_t)n * p, q.b_sb, q.b_sc);
    strides(C_case, (int64_t)m * p, q.c_sb, q.c_sc);
    // Which of the grid's (batch, channel) axes some operand actually varies
    // over; axes no operand varies over only repeat the same product.
    const bool any_b = (A_case & 1) || (B_case & 1) || (C_case & 1);
    const bool any_c = (A_case & 2) || (B_case & 2) || (C_case & 2);
    q.nbatch = any_b ? batch : 1;
    q.channels = any_c ? channels : 1;
    float mult = 1.0f;
    if (!any_b) mult *= (float)batch;
    if (!any_c) mult *= (float)channels;
    // C receives several products when an axis is iterated but C does not
    // vary over it: those are summed (the reference's atomicAdd).
    const bool c_reduces = (q.nbatch > 1 && !(C_case & 1)) || (q.channels > 1 && !(C_case & 2));
    q.alpha = scale * (backward ? mult : 1.0f);
    if (!backward) {
        q.mode = tc::EPI_ASSIGN;
        if (c_reduces) return MLE_ERR_UNSUPPORTED;  // racing assignments in the reference
    } else {
        q.mode = c_reduces ? tc::EPI_ATOMIC : tc::EPI_ACCUM;
    }
    // A reduction over batch rows that are contiguous in both operands folds
    // into K: C[m,p] += sum_z A_z^T B_z with A,B [z][n][*] row-major is one
    // GEMM with K = z*n (the Linear dW case of Engine/engine.cu:3558).
    if (backward && variant == MLE_GEMM_ATB && C_case == 0 && A_case == 3 && B_case == 3) {
        q.K = (int)((int64_t)batch * channels * n);
        q.nbatch = 1;
        q.channels = 1;
        q.a_sb = q.a_sc = q.b_sb = q.b_sc = q.c_sb = q.c_sc = 0;
        q.mode = tc::EPI_ACCUM;
        q.alpha = scale;
        return run_gemm(q, as_stream(stream));
    }
    // Broadcast B with full A and C folds the batch into M (Linear forward /
    // dX: Engine/engine.cu:3538,3552).
    if (!a_t && A_case == 3 && B_case == 0 && C_case == 3) {
        q.M = (int)((int64_t)batch * channels * m);
        q.nbatch = 1;
        q.channels = 1;
        q.a_sb = q.a_sc = q.b_sb = q.b_sc = q.c_sb = q.c_sc = 0;
        q.mode = backward ? tc::EPI_ACCUM : tc::EPI_ASSIGN;
        q.alpha = scale;
        return run_gemm(q, as_stream(stream));
    }
    return run_gemm(q, as_stream(stream));
}

int mle_linear_fwd(const float* X, const float* W, const float* bias, float* Y, int64_t rows, int in_features,
                   int out_features, mle_stream_t stream) {
    if (!X || !W || !Y || rows < 0 || in_features <= 0 || out_features <= 0) return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    return mle_gemm(X, W, Y, bias, 1, rows, out_features, in_features, in_features, out_features, out_features, 0, 0, 0,
                    0, 0, 1.0f, 0.0f, stream);
}

int mle_linear_bwd(const float* X, const float* W, const float* dY, float* dX, float* dW, float* dB, int64_t rows,
                   int in_features, int out_features, mle_stream_t stream) {
    if ((dW && !X) || !W || !dY || rows < 0 || in_features <= 0 || out_features <= 0) return MLE_ERR_ARG;
    if (rows == 0) return MLE_OK;
    int s;
    if (dX) {
        // dX[rows, in] += dY[rows, out] * W[in, out]^T
        s = mle_gemm(dY, W, dX, nullptr, 1, rows, in_features, out_features, out_features, out_features, in_features, 0,
                     0, 0, 0, 1, 1.0f, 1.0f, stream);
        if (s) return s;
    }
    // dW[in, out] += X[rows, in]^T * dY[rows, out], with dB[out] += the
    // column sums of dY taken from the same product's dY tiles
    if (dW) {
        if (rows > 0x7fffffffLL) return MLE_ERR_UNSUPPORTED;
        GemmProblem q = linear_problem(X, dY, dW, nullptr, in_features, out_features, (int)rows, in_features,
                                       out_features, out_features, 1, 0, tc::EPI_ACCUM);
        q.colsum = dB;
        g_last_kpl = 0;  // set again if the product runs on the tensor cores
        g_last_colsum = 0;
        return run_gemm(q, as_stream(stream));
    }
    if (dB) return mle_bias_grad(dY, dB, rows, out_features, 1.0f, stream);
    return MLE_OK;
}

}  // extern "C"
