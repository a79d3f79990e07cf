// Attention with the column softmax, the score matrices kept on chip.
//
// Included by gemm_tcgen05.cu (namespace mle), after the tcgen05/TMA device
// helpers and the tensor-map encoders it uses.
//
// The reference materialises scale * Q K^T, its column softmax P and, in
// the backward, dP and dS as [B, H, Sq, Sk] tensors (MultiHeadAttention's
// Headify / BMMABT / Scale / SOFTMAX type 1 / BMM chain,
// Engine/transformer.cu:647-675, and the column kernels of
// Engine/kernels.cu:2134-2235).  Here no score matrix reaches HBM; the
// column softmax is carried by two numbers per key, its max m over the
// queries (masked entries included, as the reference's SoftMask takes it)
// and its inverse sum 1/l, and every probability is recomputed from them:
//   forward   1. attn_keys_kernel<0> without P (keys on the TMEM lanes):
//                m and 1/l per key
//             2. <FA_FWD>, queries on the lanes: per block of 128 queries and
//                chunk of 64 keys, S = Q K^T (tcgen05), P = exp(scale S - m)/l
//                written back into TMEM in place, O += P V with P as the
//                TMEM operand of the next product
//   backward  3. <FA_BWD_KEYS>, keys on the lanes: per block of 128 keys and
//                chunk of 64 queries, S^T and dP^T = V dO^T, P, the column
//                dot d = sum_q P dP (thread-local: a thread owns one key), and
//                dV += P^T dO; for the mathematical key gradient a second
//                pass forms dS^T = scale P (dP - d) and dK += dS^T Q
//             4. <FA_BWD_ROWS>, queries on the lanes: S and dP again,
//                dS = scale P (dP - d[key]) in place, dQ += dS K, and for the
//                reference's key gradient Z += dS Q, whose rows are indexed
//                by key (BMMABT's backward reads dS's memory as [Sk, Sq]; with
//                Sq == Sk that is dS itself), stored transposed into dK's
//                head block as the reference's bcmmT writes it.
// Each kernel is persistent (one CTA per SM walks the (batch, head,
// 128-row block) units) and warp-specialised: warp 0 streams each unit's
// fixed operands and its chunk operands through a shared-memory ring with
// TMA that runs on across units, so the next unit's copies overlap this
// unit's work, warp 1 issues the MMAs (the next
// chunk's scores before this chunk's accumulating product, so the tensor
// cores run while the epilogue warps exponentiate), warps 2-17 own the TMEM
// lane quarters (four warps each, one per 16 of a chunk's 64 columns).  The
// accumulators stay in TMEM until a unit's last chunk, in two sets that
// alternate between units, so a unit's stores overlap the next one's
// products.
namespace tc {

constexpr int FA_FWD = 0, FA_BWD_KEYS = 1, FA_BWD_ROWS = 2;
constexpr int FA_CH = 64;         // chunk: keys (FWD, BWD_ROWS) or queries (BWD_KEYS)
constexpr int FA_SKMAX = 512;     // keys whose statistics a CTA stages in shared memory
constexpr int FA_EPI_WARPS = 16;                     // four per TMEM lane quarter
constexpr int FA_QW = FA_EPI_WARPS / 4;              // warps sharing a lane quarter
constexpr int FA_COLS = FA_CH / FA_QW;               // a chunk's columns per warp
constexpr int FA_EPI_THREADS = 32 * FA_EPI_WARPS;
constexpr int FA_THREADS = 64 + FA_EPI_THREADS;      // producer, MMA issuer, epilogue warps
static_assert(FA_COLS == 16, "the epilogue moves 16 TMEM columns per access");

struct FlashParams {
    CUtensorMap fix[2];  // per-CTA operands, 128 rows, K-major
    CUtensorMap ch[4];   // per-chunk operands, FA_CH rows (K-major or MN-major)
    const float* stats;  // column max [B*H*Sk], then inverse column sum [B*H*Sk]
    float* dvec;         // sum_q P dP per key [B*H*Sk] (written by BWD_KEYS, read by BWD_ROWS)
    float* out0;         // FWD: O; BWD_KEYS: dV; BWD_ROWS: dQ
    float* out1;         // BWD_KEYS (true key gradient): dK; BWD_ROWS (reference key gradient): dK
    int64_t o0b, o0h, o0s, o1b, o1h, o1s;  // element strides per batch, head, row
    int64_t units;       // (batch, head, 128-row block) units, walked persistently
    int H, Sq, Sk;
    int blocks;          // 128-row blocks per (batch, head)
    int nchunks;         // chunks per pass
    float scale;
    int causal, acc0, acc1, two_pass, ref_keys, round;
};

template <int KIND, int HD>
struct FlashSmem {
    static constexpr int KBL = HD / 32;                       // 32-float k-blocks of a row
    static constexpr int NFIX = KIND == FA_FWD ? 1 : 2;
    static constexpr int FIX_BYTES = 128 * HD * 4;
    static constexpr int TILE = FA_CH * HD * 4;               // one chunk operand
    static constexpr int NPOS = KIND == FA_FWD ? 2 : (KIND == FA_BWD_KEYS ? 3 : 4);
    static constexpr int NS = KIND == FA_FWD ? 4 : (KIND == FA_BWD_KEYS ? 3 : 2);  // ring slots
    static constexpr int SLOT = NPOS * TILE;
    static constexpr int RING = NFIX * FIX_BYTES;
    static constexpr int STAT = RING + NS * SLOT;
    // per key (FWD, BWD_ROWS): {m log2 e - log2(1/l), d}
    static constexpr int NSTAT = KIND == FA_BWD_KEYS ? 0 : FA_SKMAX * 8;
    static constexpr int RED = STAT + NSTAT;  // column-dot partials: [unit parity][column group][128]
    static constexpr int BAR = RED + 2 * FA_QW * 128 * 4;
    // full[NS], empty[NS], fixed_full, fixed_empty, s_full[2], epi_done[2],
    // acc_done[2], acc_free[2], drain
    static constexpr int NBARS = 2 * NS + 11;
    static constexpr int TOTAL = BAR + NBARS * 8 + 16 + 1024;  // + TMEM slot, abort flag, alignment
    static constexpr uint32_t TMEM_COLS = KIND == FA_FWD ? 256 : 512;
    // TMEM columns: score buffers S[2] (and dP[2]), then two sets of
    // accumulators (unit parity), each {ACC0, ACC1 = ACC0 + HD}
    static constexpr uint32_t SB0 = 0;
    static constexpr uint32_t PB0 = 2 * FA_CH;
    static constexpr uint32_t ACC_BASE = KIND == FA_FWD ? 2 * FA_CH : 4 * FA_CH;
    static constexpr uint32_t ACC_STRIDE = KIND == FA_FWD ? HD : 2 * HD;
    static_assert(ACC_BASE + 2 * ACC_STRIDE <= TMEM_COLS, "TMEM columns");
};

__device__ __forceinline__ void mma_tf32_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// fp32 -> tf32 operand bits: with `round`, to nearest (ties away from zero)
// at the 10-bit mantissa, as integer arithmetic on the bit pattern (the
// carry moves into the exponent when the mantissa overflows); else the
// bits as they are (the tensor cores ignore the low 13)
__device__ __forceinline__ uint32_t tf32_bits(float x, int round) {
    const uint32_t u = __float_as_uint(x);
    return round ? (u + 0x1000u) & 0xffffe000u : u;
}

template <int KIND, int HD>
__global__ void __launch_bounds__(FA_THREADS, 1) attn_flash_kernel(const __grid_constant__ FlashParams p) {
    using L = FlashSmem<KIND, HD>;
    constexpr int KBL = L::KBL;
    extern __shared__ uint8_t smem_raw[];
    // aligned by pointer arithmetic on the shared array, so that the
    // compiler keeps the address space (shared loads, not generic ones)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* fixs = smem;
    uint8_t* ring = smem + L::RING;
    float2* kst = reinterpret_cast<float2*>(smem + L::STAT);
    float* red = reinterpret_cast<float*>(smem + L::RED);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR);
    uint64_t* empty = full + L::NS;
    uint64_t* fixed_full = empty + L::NS;
    uint64_t* fixed_empty = fixed_full + 1;
    uint64_t* s_full = fixed_empty + 1;
    uint64_t* epi_done = s_full + 2;
    uint64_t* acc_done = epi_done + 2;
    uint64_t* acc_free = acc_done + 2;
    uint64_t* drain = acc_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    // scalar parameters in registers: reads through a reference into the
    // parameter space would be repeated after every shared-memory access
    const int Sq = p.Sq, Sk = p.Sk, H = p.H, blocks = p.blocks, nchunks = p.nchunks;
    const int causal = p.causal, two_pass = p.two_pass, ref_keys = p.ref_keys, round = p.round;
    const int acc_out0 = p.acc0, acc_out1 = p.acc1;
    const float scale = p.scale;
    const int64_t units = p.units;
    const float* stats = p.stats;
    float* dvec = p.dvec;
    float* out0 = p.out0;
    float* out1 = p.out1;
    const int64_t o0b = p.o0b, o0h = p.o0h, o0s = p.o0s, o1b = p.o1b, o1h = p.o1h, o1s = p.o1s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nk = units / blocks * Sk;     // B * H * Sk
    // unit u: (batch b, head h, 128-row block starting at row0); bh = b * H + h
    auto coords = [&](int64_t u, int& b, int& h, int& row0, int64_t& bh) {
        row0 = (int)(u % blocks) * 128;
        bh = u / blocks;
        h = (int)(bh % H);
        b = (int)(bh / H);
    };
    // chunks of a unit: [cb, cb + nc) in each pass.  Causal masking zeroes
    // whole chunks (queries below a key block's first key; keys above a
    // query block's last query), which are left out; one is kept at least,
    // so that every unit writes its accumulators.
    auto unit_chunks = [&](int row0, int& cb, int& nc) {
        cb = 0;
        int ce = nchunks;
        if (causal) {
            if (KIND == FA_BWD_KEYS) {
                cb = row0 / FA_CH < nchunks ? row0 / FA_CH : nchunks - 1;
            } else {
                const int qmax = row0 + 127 < Sq ? row0 + 127 : Sq - 1;
                ce = qmax / FA_CH + 1 < nchunks ? qmax / FA_CH + 1 : nchunks;
            }
        }
        nc = ce - cb;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(fixed_full, 1);
        mbar_init(fixed_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&epi_done[i], FA_EPI_WARPS);
            mbar_init(&acc_done[i], 1);
            mbar_init(&acc_free[i], FA_EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < L::NFIX; ++i)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.fix[i])) : "memory");
        for (int i = 0; i < 4; ++i)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.ch[i])) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // inputs (and the statistics of the preceding kernel) are read only from
    // here on; the next kernel may start once every CTA holds its TMEM
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            // per unit: its fixed operands (once the previous unit's last
            // score products have read the buffer), then its chunks through
            // the ring, which runs on across units
            uint32_t g = 0;
            int it = 0, fixed_it = -1;
            int64_t last = -1;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++it) {
                int b, h, row0;
                int64_t bh;
                coords(u, b, h, row0, bh);
                int cb, nc;
                unit_chunks(row0, cb, nc);
                const int nv = nc * (two_pass ? 2 : 1);
                if (it > 0 && !wait_bounded(fixed_empty, (uint32_t)(it - 1) & 1u, abort_flag)) break;
                mbar_arrive_expect_tx(fixed_full, (uint32_t)(L::NFIX * L::FIX_BYTES));
                for (int f = 0; f < L::NFIX; ++f)
#pragma unroll
                    for (int j = 0; j < KBL; ++j)
                        tma_load_4d(&p.fix[f], fixed_full, fixs + f * L::FIX_BYTES + j * 128 * 128, 32 * j, row0,
                                    h, b);
                fixed_it = it;
                for (int v = 0; v < nv; ++v, ++g) {
                    const int s = (int)(g % L::NS);
                    if (!wait_bounded(&empty[s], ((g / L::NS) & 1u) ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const int c = cb + v % nc;
                    const bool pass2 = v >= nc;
                    // chunk maps landing in positions 0.. of the slot
                    int maps[4] = {0, 1, 2, 3};
                    int n = L::NPOS;
                    if (KIND == FA_BWD_KEYS && pass2) maps[2] = 3;  // Q (MN-major) instead of dO
                    if (KIND == FA_BWD_ROWS && !ref_keys) n = 3;
                    uint8_t* slot = ring + s * L::SLOT;
                    mbar_arrive_expect_tx(&full[s], (uint32_t)(n * L::TILE));
                    for (int i = 0; i < n; ++i)
#pragma unroll
                        for (int j = 0; j < KBL; ++j)
                            tma_load_4d(&p.ch[maps[i]], &full[s], slot + i * L::TILE + j * FA_CH * 128, 32 * j,
                                        c * FA_CH, h, b);
                    last = g;
                }
            }
            if (*abort_flag) {
                // the copies in flight land before the CTA leaves
                if (fixed_it >= 0) drain_wait(fixed_full, (uint32_t)fixed_it & 1u);
                for (int64_t v = last - L::NS + 1 < 0 ? 0 : last - L::NS + 1; v <= last; ++v)
                    drain_wait(&full[v % L::NS], (uint32_t)(v / L::NS) & 1u);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------- MMA issuer -------------------------------
            // D = f32, A = B = tf32; scores: both K-major, N = FA_CH; the
            // accumulating products: A in TMEM, B MN-major, N = HD
            constexpr uint32_t kScore =
                (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(FA_CH >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
            constexpr uint32_t kAcc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                      ((uint32_t)(128 >> 4) << 24);
            const uint32_t fa = smem_u32(fixs);
            uint32_t last_g = 0;  // the current unit's last chunk
            // S (or S^T) into score buffer g & 1, and dP (or dP^T) beside it;
            // the chunk's operands have landed
            auto issue_scores = [&](uint32_t g) {
                const int s = (int)(g % L::NS);
                const uint32_t slot = smem_u32(ring + s * L::SLOT);
                const uint32_t bb = g & 1u;
#pragma unroll
                for (int j = 0; j < KBL; ++j)
#pragma unroll
                    for (int k8 = 0; k8 < 4; ++k8)
                        mma_tf32(tmem + L::SB0 + bb * FA_CH, kmajor_desc(fa + j * 128 * 128, k8),
                                 kmajor_desc(slot + j * FA_CH * 128, k8), kScore, (j | k8) ? 1u : 0u);
                if (KIND != FA_FWD) {
#pragma unroll
                    for (int j = 0; j < KBL; ++j)
#pragma unroll
                        for (int k8 = 0; k8 < 4; ++k8)
                            mma_tf32(tmem + L::PB0 + bb * FA_CH, kmajor_desc(fa + L::FIX_BYTES + j * 128 * 128, k8),
                                     kmajor_desc(slot + L::TILE + j * FA_CH * 128, k8), kScore, (j | k8) ? 1u : 0u);
                }
                mma_commit(&s_full[bb]);
                // the unit's last products reading the fixed operands: the
                // next unit's may be copied in once they retire
                if (g == last_g) mma_commit(fixed_empty);
            };
            auto scores = [&](uint32_t g) -> bool {
                if (!wait_bounded(&full[g % L::NS], (g / L::NS) & 1u, abort_flag)) return false;
                tc_fence_after();
                issue_scores(g);
                return true;
            };
            // Waits for the epilogue to finish chunk g while issuing chunk
            // g + 1's scores as soon as its operands land (when `next`): the
            // accumulating product of chunk g, which frees its ring slot,
            // never waits for the next chunk's copies.  Bounded like
            // wait_bounded.
            auto wait_epi = [&](uint32_t g, bool next, bool& next_issued) -> bool {
                uint64_t t0 = 0;
                for (uint32_t k = 0;; ++k) {
                    if (next && !next_issued && mbar_test_wait(&full[(g + 1) % L::NS], ((g + 1) / L::NS) & 1u)) {
                        tc_fence_after();
                        issue_scores(g + 1);
                        next_issued = true;
                    }
                    if (mbar_test_wait(&epi_done[g & 1u], (g >> 1) & 1u)) return true;
                    // leave the issue slots to the epilogue warps sharing this scheduler
                    __nanosleep(64);
                    if ((k & 127u) == 127u) {
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
            };
            // D += A (TMEM columns a..a+FA_CH) x B (MN-major tile at bslot)
            auto accumulate = [&](uint32_t d, uint32_t a, uint32_t bslot, bool first) {
#pragma unroll
                for (int kk = 0; kk < FA_CH / 8; ++kk)
                    mma_tf32_tmem_a(d, a + 8 * kk, mnmajor_desc(bslot, kk, FA_CH * 128), kAcc,
                                    (first && kk == 0) ? 0u : 1u);
            };
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++it) {
                int b, h, row0, cb, nc;
                int64_t bh;
                coords(u, b, h, row0, bh);
                unit_chunks(row0, cb, nc);
                const int nv = nc * (two_pass ? 2 : 1);
                last_g = g + (uint32_t)nv - 1;
                if (!wait_bounded(fixed_full, (uint32_t)it & 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int ab = it & 1;
                const uint32_t acc0 = tmem + L::ACC_BASE + (uint32_t)ab * L::ACC_STRIDE, acc1 = acc0 + HD;
                bool acc_ready = it < 2;  // the epilogue has drained unit it - 2 from this set
                if (!scores(g)) {
                    ok = false;
                    break;
                }
                bool next_issued = false;  // chunk v + 1's scores
                for (int v = 0; v < nv; ++v) {
                    const uint32_t gv = g + (uint32_t)v;
                    const bool next = v + 1 < nv;
                    // the next chunk's scores go out while the epilogue works
                    // on this one; they need the other score buffer, whose
                    // last reader (chunk v - 1's product) is already issued
                    if (v > 0) next_issued = false;
                    if (!wait_epi(gv, next, next_issued)) {
                        ok = false;
                        break;
                    }
                    if (!acc_ready) {
                        if (!wait_bounded(&acc_free[ab], (uint32_t)((it >> 1) - 1) & 1u, abort_flag)) {
                            ok = false;
                            break;
                        }
                        acc_ready = true;
                    }
                    tc_fence_after();
                    const int s = (int)(gv % L::NS);
                    const uint32_t slot = smem_u32(ring + s * L::SLOT);
                    const uint32_t bb = gv & 1u;
                    if (KIND == FA_FWD) {
                        accumulate(acc0, tmem + L::SB0 + bb * FA_CH, slot + L::TILE, v == 0);  // O += P V
                    } else if (KIND == FA_BWD_KEYS) {
                        if (v < nc)  // dV += P^T dO
                            accumulate(acc0, tmem + L::SB0 + bb * FA_CH, slot + 2 * L::TILE, v == 0);
                        else  // dK += dS^T Q
                            accumulate(acc1, tmem + L::PB0 + bb * FA_CH, slot + 2 * L::TILE, v == nc);
                    } else {
                        // dQ += dS K; reference key gradient: Z += dS Q
                        accumulate(acc0, tmem + L::PB0 + bb * FA_CH, slot + 2 * L::TILE, v == 0);
                        if (ref_keys) accumulate(acc1, tmem + L::PB0 + bb * FA_CH, slot + 3 * L::TILE, v == 0);
                    }
                    mma_commit(&empty[s]);  // the slot's products (scores and this one) have read it
                    if (next && !next_issued) {
                        if (!scores(gv + 1)) {
                            ok = false;
                            break;
                        }
                    }
                    next_issued = true;
                }
                if (!ok) break;
                g += (uint32_t)nv;
                mma_commit(&acc_done[ab]);
            }
            if (!ok) {
                mma_commit(drain);  // the issued MMAs retire before TMEM is released
                drain_wait(drain, 0);
            }
        }
        __syncwarp();
    } else {
        // ------------------------- epilogue warps 2-17 ------------------------
        // four warps per TMEM lane quarter, each taking 16 of a chunk's 64
        // columns (and 16 of an accumulator row's HD columns).  Every warp
        // walks every unit and chunk and reaches the same named barriers, also
        // after a timed-out wait (it then skips the work), so none waits for
        // a warp that left.
        const int quarter = warp & 3;
        const int ch = (warp - 2) >> 2;     // column group
        const int r = quarter * 32 + lane;  // TMEM lane = row of the 128-row block
        const uint32_t lanes = tmem + ((uint32_t)(quarter * 32) << 16);
        const int et = threadIdx.x - 64;
        // exp(scale s - m) / l = exp2(s * c2 - mm), mm = m log2 e - log2(1/l)
        const float c2 = scale * kLog2e;
        // a unit's per-key statistics are read from global memory one unit
        // ahead (its loads in flight while the previous unit runs): BWD_KEYS
        // the thread's key, else keys et and et + 256 of the head
        constexpr int NPF = (FA_SKMAX + FA_EPI_THREADS - 1) / FA_EPI_THREADS;  // keys per thread
        float pf[3 * NPF];
#pragma unroll
        for (int i = 0; i < NPF; ++i) {
            pf[3 * i] = 0.f;
            pf[3 * i + 1] = 1.f;
            pf[3 * i + 2] = 0.f;
        }
        auto fetch = [&](int64_t u) {
            if (u >= units) return;
            int b, h, row0;
            int64_t bh;
            coords(u, b, h, row0, bh);
            if (KIND == FA_BWD_KEYS) {
                const int key = row0 + r;
                if (key < Sk) {
                    pf[0] = stats[bh * Sk + key];
                    pf[1] = stats[nk + bh * Sk + key];
                }
            } else {
#pragma unroll
                for (int i = 0; i < NPF; ++i) {
                    const int k = et + i * FA_EPI_THREADS;
                    if (k < Sk) {
                        pf[3 * i] = stats[bh * Sk + k];
                        pf[3 * i + 1] = stats[nk + bh * Sk + k];
                        if (KIND == FA_BWD_ROWS) pf[3 * i + 2] = dvec[bh * Sk + k];
                    }
                }
            }
        };
        fetch(blockIdx.x);
        uint32_t g = 0;
        int it = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < units; u += gridDim.x, ++it) {
            int b, h, row0;
            int64_t bh;
            coords(u, b, h, row0, bh);
            float cur[3 * NPF];
#pragma unroll
            for (int i = 0; i < 3 * NPF; ++i) cur[i] = pf[i];
            fetch(u + gridDim.x);
            if (KIND != FA_BWD_KEYS) {
                // the previous unit's statistics are no longer read
                asm volatile("bar.sync 1, %0;" ::"n"(FA_EPI_THREADS) : "memory");
#pragma unroll
                for (int i = 0; i < NPF; ++i) {
                    const int k = et + i * FA_EPI_THREADS;
                    if (k < Sk) kst[k] = make_float2(cur[3 * i] * kLog2e - log2f(cur[3 * i + 1]), cur[3 * i + 2]);
                }
                asm volatile("bar.sync 1, %0;" ::"n"(FA_EPI_THREADS) : "memory");
            }
            const int key_r = row0 + r;  // BWD_KEYS: this thread's key; else its query
            float kmm = 0.f, dsum = 0.f;
            if (KIND == FA_BWD_KEYS && key_r < Sk) kmm = cur[0] * kLog2e - log2f(cur[1]);
            // the column dot over every query: the partial sums of the four column groups
            float* rd = red + (it & 1) * FA_QW * 128;
            auto combine_dsum = [&]() {
                rd[ch * 128 + r] = dsum;
                asm volatile("bar.sync 2, %0;" ::"n"(FA_EPI_THREADS) : "memory");
                dsum = 0.f;
#pragma unroll
                for (int w = 0; w < FA_QW; ++w) dsum += rd[w * 128 + r];
            };
            int cb, nc;
            unit_chunks(row0, cb, nc);
            const int nv = nc * (two_pass ? 2 : 1);
            for (int v = 0; v < nv; ++v) {
                const uint32_t gv = g + (uint32_t)v;
                const uint32_t bb = gv & 1u;
                ok = __all_sync(0xffffffffu, ok && wait_bounded(&s_full[bb], (gv >> 1) & 1u, abort_flag));
                if (KIND == FA_BWD_KEYS && v == nc) combine_dsum();  // two passes: pass 1 is complete
                if (!ok) continue;
                tc_fence_after();
                const int c = cb + v % nc;
                const bool pass2 = v >= nc;
                const uint32_t col = (uint32_t)(ch * FA_COLS);
                const int i0 = c * FA_CH + (int)col;  // first key (FWD, BWD_ROWS) or query (BWD_KEYS) of the columns
                uint32_t sr[FA_COLS], pr[FA_COLS], o[FA_COLS];
                tmem_ld16(lanes + L::SB0 + bb * FA_CH + col, sr);
                if (KIND != FA_FWD) tmem_ld16(lanes + L::PB0 + bb * FA_CH + col, pr);
                bool all_live;
                if (KIND == FA_BWD_KEYS) all_live = key_r < Sk && i0 + FA_COLS <= Sq && !(causal && key_r > i0);
                else all_live = key_r < Sq && i0 + FA_COLS <= Sk && !(causal && i0 + FA_COLS - 1 > key_r);
                auto body = [&](auto checked) {
                    constexpr bool CHECK = decltype(checked)::value;
#pragma unroll
                    for (int jh = 0; jh < FA_COLS; jh += 16) {
                    // 16 columns' statistics first: independent shared loads
                    float cmm[16], cd[16];
                    if (KIND != FA_BWD_KEYS) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float2 t = kst[i0 + jh + j < Sk ? i0 + jh + j : 0];
                            cmm[j] = t.x;
                            cd[j] = t.y;
                        }
                    }
#pragma unroll
                    for (int j = jh; j < jh + 16; ++j) {
                        bool live = true;
                        if (CHECK) {
                            // bitwise, so that the test is selects rather than branches
                            const int q = KIND == FA_BWD_KEYS ? i0 + j : key_r;
                            const int key = KIND == FA_BWD_KEYS ? key_r : i0 + j;
                            live = (q < Sq) & (key < Sk) & ((causal == 0) | (key <= q));
                        }
                        const float mm = KIND == FA_BWD_KEYS ? kmm : cmm[j - jh];
                        const float dk = KIND == FA_BWD_KEYS ? 0.f : cd[j - jh];
                        float pv = exp2_approx(fmaf(__uint_as_float(sr[j]), c2, -mm));
                        if (CHECK) pv = live ? pv : 0.f;
                        if (KIND == FA_FWD) {
                            o[j] = tf32_bits(pv, round);
                        } else if (KIND == FA_BWD_KEYS) {
                            const float dp = __uint_as_float(pr[j]);
                            if (!pass2) {
                                dsum = fmaf(pv, dp, dsum);
                                o[j] = tf32_bits(pv, round);
                            } else {
                                o[j] = tf32_bits(scale * pv * (dp - dsum), round);
                            }
                        } else {
                            o[j] = tf32_bits(scale * pv * (__uint_as_float(pr[j]) - dk), round);
                        }
                    }
                    }
                };
                if (all_live) body(std::false_type());
                else body(std::true_type());
                // P (or P^T) replaces S; dS (or dS^T) replaces dP
                const bool to_s = KIND == FA_FWD || (KIND == FA_BWD_KEYS && !pass2);
                tmem_st16(lanes + (to_s ? L::SB0 : L::PB0) + bb * FA_CH + col, o);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&epi_done[bb]);
            }
            g += (uint32_t)nv;
            if (KIND == FA_BWD_KEYS && !two_pass) combine_dsum();
            const int ab = it & 1;
            ok = __all_sync(0xffffffffu, ok && wait_bounded(&acc_done[ab], (uint32_t)(it >> 1) & 1u, abort_flag));
            if (ok && ch < HD / 16) {
                tc_fence_after();
                const uint32_t cc = (uint32_t)(ch * 16);  // this warp's 16 accumulator columns
                const uint32_t acc0 = L::ACC_BASE + (uint32_t)ab * L::ACC_STRIDE, acc1 = acc0 + HD;
                // 16 accumulated floats of one row leave per thread
                auto store_row = [&](uint32_t acc_col, float* dst, bool live, int accum) {
                    uint32_t a[16];
                    tmem_ld16(lanes + acc_col + cc, a);
                    if (!live) return;
                    float4* d4 = reinterpret_cast<float4*>(dst + cc);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float4 x = make_float4(__uint_as_float(a[4 * j]), __uint_as_float(a[4 * j + 1]),
                                               __uint_as_float(a[4 * j + 2]), __uint_as_float(a[4 * j + 3]));
                        if (accum) {
                            const float4 y = d4[j];
                            x.x += y.x;
                            x.y += y.y;
                            x.z += y.z;
                            x.w += y.w;
                        }
                        d4[j] = x;
                    }
                };
                const int row = key_r;
                if (KIND == FA_FWD) {
                    store_row(acc0, out0 + (int64_t)b * o0b + (int64_t)h * o0h + (int64_t)row * o0s,
                              row < Sq, 0);
                } else if (KIND == FA_BWD_KEYS) {
                    const bool live = row < Sk;
                    if (live && ch == 0) dvec[bh * Sk + row] = dsum;
                    store_row(acc0, out0 + (int64_t)b * o0b + (int64_t)h * o0h + (int64_t)row * o0s, live,
                              acc_out0);
                    if (two_pass)
                        store_row(acc1, out1 + (int64_t)b * o1b + (int64_t)h * o1h + (int64_t)row * o1s,
                                  live, acc_out1);
                } else {
                    store_row(acc0, out0 + (int64_t)b * o0b + (int64_t)h * o0h + (int64_t)row * o0s,
                              row < Sq, acc_out0);
                    if (ref_keys) {
                        // Z[i, d] lands at row d * (Sk / HD) + i / HD, column i % HD
                        // of the head's block: a warp's 32 consecutive i fill 32
                        // consecutive floats of one row
                        float* base = out1 + (int64_t)b * o1b + (int64_t)h * o1h;
                        const int per = Sk / HD;
                        uint32_t a[16];
                        tmem_ld16(lanes + acc1 + cc, a);
                        if (row < Sq) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int d = (int)cc + j;
                                float* dst = base + (int64_t)(d * per + row / HD) * o1s + (row % HD);
                                const float x = __uint_as_float(a[j]);
                                *dst = acc_out1 ? *dst + x : x;
                            }
                        }
                    }
                }
            }
            // this set of accumulators may take unit it + 2
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[ab]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS)
                     : "memory");
    }
}

}  // namespace tc

namespace {

template <int KIND, int HD>
int launch_flash(const tc::FlashParams& prm, cudaStream_t st) {
    using L = tc::FlashSmem<KIND, HD>;
    static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
    static_assert(sizeof(tc::FlashParams) <= 4000, "kernel parameter space");
    auto kern = tc::attn_flash_kernel<KIND, HD>;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) != cudaSuccess)
            return launch_status();
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    // persistent: one CTA per SM walks the units
    cfg.gridDim = dim3((unsigned)std::min<int64_t>(prm.units, kSMs));
    cfg.blockDim = dim3(tc::FA_THREADS);
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

template <int KIND>
int launch_flash_hd(int hd, const tc::FlashParams& prm, cudaStream_t st) {
    if (hd == 32) return launch_flash<KIND, 32>(prm, st);
    if (hd == 64) return launch_flash<KIND, 64>(prm, st);
    return MLE_ERR_UNSUPPORTED;
}

// (hd, S, H, B) view of a token- or head-major operand, boxes of `rows` rows
bool flash_map(CUtensorMap* m, const float* base, int hd, int S, int H, int B, int64_t sb, int64_t sh, int64_t ss,
               int rows, bool mn_major) {
    const int64_t dims[4] = {hd, S, H, B}, strides[3] = {ss, sh, sb};
    const int box[4] = {32, rows, 1, 1};
    return tc::encode_map(m, base, dims, strides, box,
                          mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B, 4,
                          operand_type());
}

}  // namespace

bool attn_flash_supported(int Sq, int Sk, int hd, int64_t BH, int key_mode) {
    if (Sq <= 0 || Sq > 256 || Sk <= 0 || Sk > tc::FA_SKMAX || (hd != 32 && hd != 64)) return false;
    if (key_mode == MLE_KEYGRAD_REFERENCE && !(Sq == Sk && Sk % hd == 0)) return false;
    if (BH * ((std::max(Sq, Sk) + 127) / 128) > 0x7fffffff || BH * Sk * 2 > ((int64_t)1 << 40)) return false;
    return tc::get_encode() != nullptr;
}

int run_attn_flash_fwd(const float* Q, const float* K, const float* V, float* O, float* stats, int B, int H, int Sq,
                       int Sk, int hd, int64_t qb, int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks,
                       float scale, int causal, cudaStream_t st) {
    if (!attn_flash_supported(Sq, Sk, hd, (int64_t)B * H, MLE_KEYGRAD_TRUE)) return MLE_ERR_UNSUPPORTED;
    tc::FlashParams prm;
    memset(&prm, 0, sizeof(prm));
    if (!flash_map(&prm.fix[0], Q, hd, Sq, H, B, qb, qh, qs, 128, false) ||
        !flash_map(&prm.ch[0], K, hd, Sk, H, B, kb, kh, ks, tc::FA_CH, false) ||
        !flash_map(&prm.ch[1], V, hd, Sk, H, B, kb, kh, ks, tc::FA_CH, true))
        return MLE_ERR_UNSUPPORTED;
    // column statistics (keys on the lanes), then O (queries on the lanes)
    int s = run_attn_keys(0, K, Q, nullptr, nullptr, B, H, Sq, Sk, hd, kb, kh, ks, qb, qh, qs, scale, causal, st,
                          stats);
    if (s) return s;
    prm.stats = stats;
    prm.out0 = O;
    prm.o0b = qb;
    prm.o0h = qh;
    prm.o0s = qs;
    prm.H = H;
    prm.Sq = Sq;
    prm.Sk = Sk;
    prm.blocks = (Sq + 127) / 128;
    prm.nchunks = (Sk + tc::FA_CH - 1) / tc::FA_CH;
    prm.scale = scale;
    prm.causal = causal;
    prm.round = g_operand_round;
    prm.units = (int64_t)B * H * prm.blocks;
    return launch_flash_hd<tc::FA_FWD>(hd, prm, st);
}

int run_attn_flash_bwd(const float* Q, const float* K, const float* V, const float* dO, const float* stats,
                       float* dvec, float* dQ, float* dK, float* dV, int B, int H, int Sq, int Sk, int hd, int64_t qb,
                       int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks, float scale, int causal,
                       int key_mode, int assign, cudaStream_t st) {
    if (!attn_flash_supported(Sq, Sk, hd, (int64_t)B * H, key_mode)) return MLE_ERR_UNSUPPORTED;
    const bool ref = key_mode == MLE_KEYGRAD_REFERENCE;
    tc::FlashParams kp, rp;
    memset(&kp, 0, sizeof(kp));
    memset(&rp, 0, sizeof(rp));
    // keys on the lanes: K, V per CTA; Q, dO (and their MN-major copies) per chunk
    if (!flash_map(&kp.fix[0], K, hd, Sk, H, B, kb, kh, ks, 128, false) ||
        !flash_map(&kp.fix[1], V, hd, Sk, H, B, kb, kh, ks, 128, false) ||
        !flash_map(&kp.ch[0], Q, hd, Sq, H, B, qb, qh, qs, tc::FA_CH, false) ||
        !flash_map(&kp.ch[1], dO, hd, Sq, H, B, qb, qh, qs, tc::FA_CH, false) ||
        !flash_map(&kp.ch[2], dO, hd, Sq, H, B, qb, qh, qs, tc::FA_CH, true) ||
        !flash_map(&kp.ch[3], Q, hd, Sq, H, B, qb, qh, qs, tc::FA_CH, true))
        return MLE_ERR_UNSUPPORTED;
    // queries on the lanes: Q, dO per CTA; K, V (and MN-major K, Q) per chunk
    if (!flash_map(&rp.fix[0], Q, hd, Sq, H, B, qb, qh, qs, 128, false) ||
        !flash_map(&rp.fix[1], dO, hd, Sq, H, B, qb, qh, qs, 128, false) ||
        !flash_map(&rp.ch[0], K, hd, Sk, H, B, kb, kh, ks, tc::FA_CH, false) ||
        !flash_map(&rp.ch[1], V, hd, Sk, H, B, kb, kh, ks, tc::FA_CH, false) ||
        !flash_map(&rp.ch[2], K, hd, Sk, H, B, kb, kh, ks, tc::FA_CH, true) ||
        !flash_map(&rp.ch[3], Q, hd, Sq, H, B, qb, qh, qs, tc::FA_CH, true))
        return MLE_ERR_UNSUPPORTED;
    kp.stats = rp.stats = stats;
    kp.dvec = rp.dvec = dvec;
    kp.H = rp.H = H;
    kp.Sq = rp.Sq = Sq;
    kp.Sk = rp.Sk = Sk;
    kp.scale = rp.scale = scale;
    kp.causal = rp.causal = causal;
    kp.round = rp.round = g_operand_round;
    kp.out0 = dV;
    kp.o0b = kb;
    kp.o0h = kh;
    kp.o0s = ks;
    kp.acc0 = (assign & 4) ? 0 : 1;
    kp.two_pass = ref ? 0 : 1;
    kp.out1 = dK;
    kp.o1b = kb;
    kp.o1h = kh;
    kp.o1s = ks;
    kp.acc1 = (assign & 2) ? 0 : 1;
    kp.blocks = (Sk + 127) / 128;
    kp.nchunks = (Sq + tc::FA_CH - 1) / tc::FA_CH;
    kp.units = (int64_t)B * H * kp.blocks;
    int s = launch_flash_hd<tc::FA_BWD_KEYS>(hd, kp, st);
    if (s) return s;
    rp.out0 = dQ;
    rp.o0b = qb;
    rp.o0h = qh;
    rp.o0s = qs;
    rp.acc0 = (assign & 1) ? 0 : 1;
    rp.ref_keys = ref ? 1 : 0;
    rp.out1 = dK;
    rp.o1b = kb;
    rp.o1h = kh;
    rp.o1s = ks;
    rp.acc1 = (assign & 2) ? 0 : 1;
    rp.blocks = (Sq + 127) / 128;
    rp.nchunks = (Sk + tc::FA_CH - 1) / tc::FA_CH;
    rp.units = (int64_t)B * H * rp.blocks;
    return launch_flash_hd<tc::FA_BWD_ROWS>(hd, rp, st);
}
