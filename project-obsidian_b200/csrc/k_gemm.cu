// k_gemm.cu -- prefill expert FFN: grouped 4-bit dequant GEMM on tcgen05.
//
// Replaces the reference's per-expert matmul_dequant_4bit dispatches
// (shaders/matmul_dequant_4bit.metal:21-66; host src/forward.rs:313-321,
// per-expert calls :219-222) and the ew_swiglu between them (ops.metal:18-22).
//
// One persistent CTA per SM walks work items (token tile of <= 64 rows, weight
// row tile of 128 rows), seventeen warps in five roles:
//   warp 0      weight producer: 1-D bulk async copies of the packed weight
//               block(s) (4608 B each, contiguous by construction of the HBM
//               layout) into a deep shared-memory ring (W);
//   warps 1-2   token-tile producer into the B ring (eight k-steps deep): for
//               gate/up, rows of the layer input gathered by source token with
//               16-byte cp.async (L2 evict-last) into the 128-byte-swizzled
//               K-major slots (zero fill for padding rows), each thread's
//               completion arriving on the stage's full barrier; for down,
//               bulk copies of the tiled H rows;
//   warps 3-4   MMA issuers (one thread each): tcgen05.mma kind::f16 with A in
//               TMEM and B in shared memory, M = 128 weight rows, N = token
//               rows, K = 16, fp32 accumulators in TMEM.  Issuer 0 owns the
//               gate chain (or the even k-slices), issuer 1 the up chain (odd
//               k-slices); two accumulator buffers let the epilogue overlap the
//               next item.  A stage and its B stage are free once both issuers'
//               commits of that k-step have arrived;
//   warps 5-12  dequantise a W stage (released as soon as it is read) straight
//               into tensor memory: two codes per bf16x2 register,
//               q = (0x4300 | n) - 128, w = fma.rn.bf16x2(q, s, b) (the correctly
//               rounded bf16 of q*s + b), written with tcgen05.st into an A stage
//               of TMEM (one weight row per TMEM lane, four A stages); each warp
//               owns the TMEM lane quarter it may access;
//   warps 13-16 epilogue: tcgen05.ld, SwiGLU (or plain), results staged in
//               shared memory in the global layout and written back with bulk
//               copies (fp32 debug output: direct stores).
// Keeping A out of shared memory leaves shared-memory bandwidth to the weight
// and token streams.  The packed words hold their codes in the nibble order
// (c0,c2,c4,c6,c1,c3,c5,c7) (set by the loader), so (w >> 4j) & 0x000F000F is
// the bf16x2 pair of columns (2j, 2j+1).
// Every mbarrier wait is bounded; a CTA that gives up records kDevTimeout,
// drains its outstanding copies (bounded), frees its TMEM and returns.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kBN = 64;  // token rows per tile (tcgen05 N <= 64 here)
constexpr int kDqWarps = 8, kEpWarps = 4;
// two MMA issuers in two warps: one thread issues a tcgen05.mma about every 50
// cycles, and every other instruction it runs between MMAs (a barrier wait, a
// branch) leaves the tensor pipe idle; two issuers feeding independent
// accumulators keep it busy (M=128, N=64, K=16 every ~32 cycles)
constexpr int kWarpW = 0, kWarpB = 1, kWarpMma = 3, kMmaWarps = 2, kWarpDq = kWarpMma + kMmaWarps,
              kWarpEp = kWarpDq + kDqWarps;
constexpr int kThreads = 32 * (kWarpEp + kEpWarps);  // 544
constexpr int kEpThreads = 32 * kEpWarps;

template <int EPI>
struct Cfg {
    static constexpr bool GATHER = EPI == kEpiSwiglu;    // token tile gathered from x rows
    static constexpr int NP = EPI == kEpiSwiglu ? 2 : 1;  // projections per tile (gate, up)
    static constexpr int W_STAGE = NP * kBlockBytes;      // packed weights of one k-step (16-byte multiple)
    // W ring: chunks of a.wchunk consecutive k-steps, one bulk copy each (a lone
    // producer thread issues roughly one copy per 0.3 us, so small copies cap
    // the weight stream well below HBM bandwidth); W_BYTES / (chunk bytes) stages
    static constexpr int W_BYTES = 6 * 4 * kBlockBytes;   // 110592
    static constexpr int SW = W_BYTES / kBlockBytes;      // barrier slots for the smallest chunk
    static constexpr int B_STAGE = kBN * 128;
    static constexpr int SA = 4;                          // A stages in TMEM
    // B stages: twice as deep as A, so the token-tile latency (a gather from L2)
    // is hidden behind eight k-steps.  One commit per k-step, to the B stage's
    // "free" barrier, also frees the A stage of that k-step; a dequant warp
    // reusing A stage (i mod SA) waits for the commit of k-step i - SA.
    static constexpr int SB = 2 * SA;
    // accumulators per buffer: gate + up, or (single projection) even + odd k-slices,
    // so consecutive MMAs always target independent accumulators
    static constexpr int ACC_COLS = 2 * kBN;              // one accumulator buffer (fp32 columns)
    static constexpr int A_COLS = NP * 32;                // one A stage: 64 bf16 per row = 32 columns
    static constexpr int A_TMEM = 2 * ACC_COLS;           // first A stage column
    static constexpr int TMEM_COLS = 512;
    static_assert(A_TMEM + SA * A_COLS <= TMEM_COLS, "tmem");
    static constexpr int STG = kBN * 256;                 // epilogue staging: 64 rows x 128 features bf16
    static constexpr int B_OFF = 0;                       // 1024-aligned tiles first
    static constexpr int STG_OFF = B_OFF + SB * B_STAGE;
    static constexpr int W_OFF = STG_OFF + 2 * STG;
    static constexpr int BAR_OFF = (W_OFF + W_BYTES + 7) / 8 * 8;
    static constexpr int N_BARS = 2 * SW + 2 * SB + 2 * SA + 4;  // (aempty unused: empty_b frees A too)
    static constexpr int SMEM = BAR_OFF + N_BARS * 8 + 32 + 1024;  // + alignment slack
};
static_assert(Cfg<kEpiSwiglu>::SMEM <= 232448, "smem");
static_assert(Cfg<kEpiBf16>::SMEM <= 232448, "smem");

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// 8 codes of one word (nibble order c0,c2,c4,c6,c1,c3,c5,c7) -> 4 bf16x2 in column order
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t s2, uint32_t b2, uint32_t* out) {
    const uint32_t magic = 0x43004300u;  // bf16x2 (128, 128)
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = bf2_fma(bf2_sub(((w >> (4 * j)) & 0x000F000Fu) | magic, magic), s2, b2);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(dst), "l"(src),
                 "r"(src_bytes), "l"(policy)
                 : "memory");
}
// the mbarrier receives one arrival when all prior cp.async of this thread complete
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

__device__ __forceinline__ bool wait_all(uint32_t bar, uint32_t parity, volatile int* abort) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

// After giving up, a producer waits (bounded) until the newest copy it issued
// into each stage of its ring has landed, so no copy targets freed memory.
__device__ __forceinline__ void drain_ring(uint32_t bar0, int stages, int issued) {
    for (int st = 0; st < stages && st < issued; ++st) {
        const int last = st + (issued - 1 - st) / stages * stages;
        const uint32_t par = (last / stages) & 1;
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(bar0 + 8 * st, par) && global_ns() - t0 < kWaitLimitNs) {
        }
    }
}

// Pipeline trace (CTA 0 only), compiled into the TRACE instances alone: the
// branch costs the MMA issuer tensor-pipe time.
template <bool TRACE>
__device__ __forceinline__ void trace_at(const GemmArgs& a, int role, int i) {
    if constexpr (TRACE)
        if (blockIdx.x == 0 && i < a.trace_n) a.trace[(size_t)role * a.trace_n + i] = global_ns();
}

template <int EPI, bool TRACE>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(GemmArgs a) {
    using C = Cfg<EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t bar_base = smem_u32(bars);
    auto full_w = [&](int s) { return bar_base + 8 * s; };
    auto empty_w = [&](int s) { return bar_base + 8 * (C::SW + s); };
    auto full_b = [&](int s) { return bar_base + 8 * (2 * C::SW + s); };
    auto empty_b = [&](int s) { return bar_base + 8 * (2 * C::SW + C::SB + s); };
    auto aready = [&](int s) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + s); };
    auto aempty = [&](int s) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + C::SA + s); };
    auto accfull = [&](int b) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + 2 * C::SA + b); };
    auto accempty = [&](int b) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + 2 * C::SA + 2 + b); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < C::SW; ++s) mbar_init(full_w(s), 1), mbar_init(empty_w(s), kDqWarps);
        // "stage free" and "accumulator full" complete on one commit from each issuer
        for (int s = 0; s < C::SB; ++s) mbar_init(full_b(s), C::GATHER ? 64 : 1), mbar_init(empty_b(s), kMmaWarps);
        for (int s = 0; s < C::SA; ++s) mbar_init(aready(s), kDqWarps), mbar_init(aempty(s), 1);
        for (int b = 0; b < 2; ++b) mbar_init(accfull(b), kMmaWarps), mbar_init(accempty(b), kEpThreads);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = *a.n_tiles * a.n_rt;
    const int KT = a.n_kt;

    const int wch = a.wchunk;                         // k-steps per weight copy
    const uint32_t wcbytes = (uint32_t)wch * C::W_STAGE;
    const int nsw = C::W_BYTES / (int)wcbytes;        // W ring stages

    if (warp == kWarpW) {
        // ---------------------------------------------- weight producer (bulk)
        // the whole warp runs the loop, one elected lane issues
        const uint64_t pol = policy_evict_first();
        int s = 0, ph = 0, issued = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            const uint8_t* wsrc =
                a.wblocks + (((size_t)tl.x * a.n_rt + rt) * KT * a.wstride + a.woff) * kBlockBytes;
            for (int kt = 0; kt < KT; kt += wch) {
                if (!wait_all(empty_w(s), ph ^ 1, abort_flag)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(full_w(s), wcbytes);
                    bulk_g2s_hint(sbase + C::W_OFF + s * wcbytes, wsrc + (size_t)kt * a.wstride * kBlockBytes, wcbytes,
                                  full_w(s), pol);
                }
                __syncwarp();
                if (lane == 0) trace_at<TRACE>(a, kTrWIssue, issued);
                ++issued;
                if (++s == nsw) s = 0, ph ^= 1;
            }
        }
        if (*abort_flag && lane == 0) drain_ring(full_w(0), nsw, issued);
        __syncwarp();
    } else if (warp == kWarpB || warp == kWarpB + 1) {
        // ----------------------------------------------- token-tile producer
        if constexpr (C::GATHER) {
            const int wb = warp - kWarpB, c = lane & 7, rsub = 4 * wb + (lane >> 3);
            const uint64_t pol = policy_evict_last();  // the rows are re-read by every row tile
            int s = 0, ph = 0, step = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int4 tl = a.tiles[item / a.n_rt];
                const int passes = tl.z >> 3;  // 8 rows per pass of the two warps
                int tok[kBN / 8];
#pragma unroll
                for (int p = 0; p < kBN / 8; ++p) tok[p] = p < passes ? a.src[tl.y + 8 * p + rsub] : -1;
                for (int kt = 0; kt < KT; ++kt, ++step) {
                    if (!wait_all(empty_b(s), ph ^ 1, abort_flag)) { ok = false; break; }
                    const uint32_t bst = sbase + C::B_OFF + s * C::B_STAGE;
#pragma unroll
                    for (int p = 0; p < kBN / 8; ++p) {
                        if (p < passes) {
                            const int j = 8 * p + rsub, t = tok[p];
                            const uint16_t* src = a.x_rows + (size_t)(t >= 0 ? t : 0) * a.x_ld + kt * kGroup + c * 8;
                            cp_async16(bst + (j >> 3) * 1024 + (j & 7) * 128 + ((c ^ (j & 7)) << 4), src,
                                       t >= 0 ? 16u : 0u, pol);
                        }
                    }
                    cp_async_arrive_noinc(full_b(s));
                    if (wb == 0 && lane == 0) trace_at<TRACE>(a, kTrBSignal, step);
                    if (++s == C::SB) s = 0, ph ^= 1;
                }
            }
            cp_async_wait_all();  // nothing may land after the CTA exits
        } else if (warp == kWarpB && lane == 0) {
            const uint64_t pol = policy_evict_last();
            int s = 0, ph = 0, issued = 0;
            for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
                const int4 tl = a.tiles[item / a.n_rt];
                const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(a.act) + (size_t)(tl.y >> 3) * 1024;
                const uint32_t bbytes = (uint32_t)tl.z * 128u;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!mbar_wait(empty_b(s), ph ^ 1, abort_flag)) break;
                    mbar_arrive_expect_tx(full_b(s), bbytes);
                    bulk_g2s_hint(sbase + C::B_OFF + s * C::B_STAGE, xsrc + (size_t)kt * a.atoms * 1024, bbytes,
                                  full_b(s), pol);
                    trace_at<TRACE>(a, kTrBSignal, issued);
                    ++issued;
                    if (++s == C::SB) s = 0, ph ^= 1;
                }
            }
            if (*abort_flag) drain_ring(full_b(0), C::SB, issued);
        }
        __syncwarp();
    } else if (warp < kWarpMma + kMmaWarps) {
        // --------------------------------------------------------- MMA issuers
        // issuer mi: gate/up -> projection mi (its own accumulator chain);
        // single projection -> k-slices kk = mi, mi + 2 into accumulator mi.
        // The whole warp runs the loop (waits, descriptor arithmetic) and one
        // elected lane issues: a loop run by lane 0 alone issues far slower.
        const int mi = warp - kWarpMma;
        int sa = 0, pha = 0, sb = 0, phb = 0, it = 0, step = 0;
        const uint32_t a_tmem0 = tmem + C::A_TMEM;
        const uint64_t b_desc0 = sw128_desc(sbase + C::B_OFF);
        const bool tr = TRACE && mi == 0 && lane == 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++it) {
            const int4 tl = a.tiles[item / a.n_rt];
            const uint32_t idesc = idesc_bf16(128, tl.z);
            const int buf = it & 1;
            if (!wait_all(accempty(buf), ((it >> 1) & 1) ^ 1, abort_flag)) break;
            tc_fence_after();
            const uint32_t dbase = tmem + buf * C::ACC_COLS + mi * kBN;
            bool ok = true;
            for (int kt = 0; kt < KT; ++kt) {
                if (!__all_sync(0xffffffffu, mbar_wait(aready(sa), pha, abort_flag) &&
                                                  mbar_wait(full_b(sb), phb, abort_flag))) {
                    ok = false;
                    break;
                }
                if (tr) trace_at<TRACE>(a, kTrMmaStart, step);
                tc_fence_after();
                if (tr) trace_at<TRACE>(a, kTrMmaFenced, step);
                // descriptors: plain adds on precomputed bases (the start address field
                // advances 16 bytes per unit; stages stay below 256 KB)
                const uint32_t abase = a_tmem0 + sa * C::A_COLS;
                const uint64_t bdesc = b_desc0 + (uint64_t)(sb * (C::B_STAGE >> 4));
                const uint32_t acc0 = kt != 0;
                if (elect_one()) {
                    if constexpr (C::NP == 2) {  // this issuer's projection: 4 k-slices
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc_mma_f16_ts(dbase, abase + mi * 32 + kk * 8, bdesc + 2 * kk, idesc, kk == 0 ? acc0 : 1u);
                    } else {  // even or odd k-slices into accumulator mi, summed by the epilogue
#pragma unroll
                        for (int kk = 0; kk < 4; kk += 2)
                            tc_mma_f16_ts(dbase, abase + (kk + mi) * 8, bdesc + 2 * (kk + mi), idesc,
                                          kk == 0 ? acc0 : 1u);
                    }
                    tc_commit(empty_b(sb));  // with the other issuer's: frees B stage sb and A stage sa
                }
                __syncwarp();
                if (tr) trace_at<TRACE>(a, kTrMmaIssued, step);
                ++step;
                if (++sa == C::SA) sa = 0, pha ^= 1;
                if (++sb == C::SB) sb = 0, phb ^= 1;
            }
            if (!ok) break;
            if (elect_one()) tc_commit(accfull(buf));
            __syncwarp();
        }
    } else if (warp < kWarpEp) {
        // ------------------------------------------------------------ dequant
        const int dw = warp - kWarpDq;           // 0..7
        const int q = warp & 3;                  // TMEM lane quarter this warp may write
        const int r = q * 32 + lane;             // weight row of the tile = TMEM lane
        const int part = dw >> 2;                // 0..1: which half of the (projections x words) of the row
        // gate/up: part = projection (its 8 words); plain: part = half of the row's 8 words
        const int p = C::NP == 2 ? part : 0;
        const int wofs = C::NP == 2 ? 0 : part * 4;  // first word of this part
        constexpr int NW = C::NP == 2 ? 8 : 4;       // words per part
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + C::A_TMEM + p * 32 + wofs * 4;
        // This CTA's k-steps in order (items x k-tiles), software-pipelined per
        // warp: the packed words of k-step i+1 are read from the W ring while
        // the TMEM store of k-step i drains; k-step i's A stage is signalled
        // ready as soon as its own store has completed.
        const int my_items = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int total = my_items * KT;
        uint32_t ws[NW], sv = 0, bv = 0;
        int ls = 0, lph = 0, lj = 0;  // W ring stage, phase and k-step in chunk of the next load
        // read the packed words (and the row's scale and bias) of k-step i; the
        // chunk's stage is released after its last k-step has been read
        auto load_w = [&](int i) -> bool {
            if (lj == 0 && !wait_all(full_w(ls), lph, abort_flag)) return false;
            if (dw == 0 && lane == 0) trace_at<TRACE>(a, kTrDqStart, i);
            const uint8_t* blk = smem + C::W_OFF + ls * wcbytes + lj * C::W_STAGE + p * kBlockBytes;
            const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
            sv = sb[r];
            bv = sb[kRowTile + r];
            // words [wofs, wofs + NW) of row r: word w lives in plane w/4 of the block
#pragma unroll
            for (int pl = 0; pl < NW / 4; ++pl) {
                const uint4 w0 = *reinterpret_cast<const uint4*>(blk + ((wofs >> 2) + pl) * 2048 + r * 16);
                ws[4 * pl] = w0.x, ws[4 * pl + 1] = w0.y, ws[4 * pl + 2] = w0.z, ws[4 * pl + 3] = w0.w;
            }
            if (++lj == wch) {
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_w(ls));  // chunk consumed: recycle early
                lj = 0;
                if (++ls == nsw) ls = 0, lph ^= 1;
            }
            return true;
        };
        bool ok = total == 0 || load_w(0);
        for (int step = 0; step < total && ok; ++step) {
            const int sa = step % C::SA;
            const uint32_t s2v = sv | (sv << 16), b2v = bv | (bv << 16);
            uint32_t v[4 * NW];
#pragma unroll
            for (int c = 0; c < NW; ++c) dequant_word(ws[c], s2v, b2v, &v[4 * c]);
            // A stage sa was last read by the MMAs of k-step (step - SA)
            const int prev = step - C::SA;
            if (prev >= 0 && !wait_all(empty_b(prev % C::SB), (prev / C::SB) & 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t at = trow + sa * C::A_COLS;
            if constexpr (NW == 8)
                tmem_st32(at, v);
            else
                tmem_st16(at, v);
            if (dw == 0 && lane == 0) trace_at<TRACE>(a, kTrDqStored, step);
            if (step + 1 < total && !load_w(step + 1)) ok = false;  // overlaps the store
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aready(sa));
            if (dw == 0 && lane == 0) trace_at<TRACE>(a, kTrDqDone, step);
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;          // TMEM lane quarter of this warp
        const int f = q * 32 + lane;     // accumulator row = weight row (feature) of the tile
        const int et = tid - 32 * kWarpEp;
        int it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            const int buf = it & 1;
            if (!wait_all(accfull(buf), (it >> 1) & 1, abort_flag)) break;
            if (et == 0) trace_at<TRACE>(a, kTrEpStart, it);
            tc_fence_after();
            const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + buf * C::ACC_COLS;
            if constexpr (EPI == kEpiF32) {
                const int nstore = min(tl.z, a.row_limit - tl.y);
                float* y = reinterpret_cast<float*>(a.out);
                for (int j0 = 0; j0 < tl.z; j0 += 16) {
                    float g[16], g1[16];
                    tmem_ld16(tq + j0, g);
                    tmem_ld16(tq + kBN + j0, g1);
                    tc_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        if (j0 + jj < nstore) y[(size_t)(tl.y + j0 + jj) * a.out_ld + rt * kRowTile + f] = g[jj] + g1[jj];
                }
                tc_fence_before();
                mbar_arrive(accempty(buf));
            } else {
                // the staging buffer of two items ago must have been read by its bulk store
                if (et == 0) bulk_wait_read1();
                named_bar_sync(1, kEpThreads);
                uint8_t* stg = smem + C::STG_OFF + buf * C::STG;
                for (int j0 = 0; j0 < tl.z; j0 += 16) {
                    float g[16], u[16];
                    tmem_ld16(tq + j0, g);
                    tmem_ld16(tq + kBN + j0, u);  // up projection, or the odd k-slices
                    if constexpr (EPI == kEpiSwiglu) {
                        tc_wait_ld();
                        // staging = two k-tile planes of H (features f>>6), swizzled like the global layout
                        const int fc = f & 63;
                        uint8_t* pl = stg + (f >> 6) * (kBN * 128) + ((fc & 7) << 1);
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int j = j0 + jj;
                            const float gv = g[jj];
                            const float hv = (gv / (1.0f + expf(-gv))) * u[jj];  // ops.metal:21
                            *reinterpret_cast<uint16_t*>(pl + (j >> 3) * 1024 + (j & 7) * 128 + (((fc >> 3) ^ (j & 7)) << 4)) =
                                f2bf(hv);
                        }
                    } else {
                        tc_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj)
                            *reinterpret_cast<uint16_t*>(stg + (j0 + jj) * 256 + f * 2) = f2bf(g[jj] + u[jj]);
                    }
                }
                tc_fence_before();
                mbar_arrive(accempty(buf));  // accumulator drained: the next item may start
                fence_proxy_async_smem();    // staging written by threads -> read by the bulk copy
                named_bar_sync(1, kEpThreads);
                if (et == 0) {
                    if constexpr (EPI == kEpiSwiglu) {
                        uint8_t* hb = reinterpret_cast<uint8_t*>(a.out);
#pragma unroll
                        for (int pln = 0; pln < 2; ++pln)
                            bulk_s2g(hb + ((size_t)(rt * 2 + pln) * a.out_atoms + (tl.y >> 3)) * 1024,
                                     sbase + C::STG_OFF + buf * C::STG + pln * (kBN * 128), (uint32_t)tl.z * 128u);
                    } else {
                        uint8_t* yb = reinterpret_cast<uint8_t*>(a.out);
                        const int nstore = min(tl.z, a.row_limit - tl.y);
                        for (int j = 0; j < nstore; ++j)
                            bulk_s2g(yb + ((size_t)(tl.y + j) * a.out_ld + rt * kRowTile) * 2,
                                     sbase + C::STG_OFF + buf * C::STG + j * 256, 256u);
                    }
                    bulk_commit();
                    trace_at<TRACE>(a, kTrEpDone, it);
                }
            }
        }
        if (et == 0) bulk_wait0();  // results are in global memory before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) tmem_dealloc(tmem, C::TMEM_COLS);
    if (tid == 0 && *abort_flag) atomicExch(a.err, kDevTimeout);
}

}  // namespace

size_t gemm_smem_bytes(int epi) {
    return epi == kEpiSwiglu ? Cfg<kEpiSwiglu>::SMEM : epi == kEpiBf16 ? Cfg<kEpiBf16>::SMEM : Cfg<kEpiF32>::SMEM;
}
int gemm_tile_rows() { return kBN; }

template <int EPI>
static cudaError_t launch_t(GemmArgs a, int num_sms, cudaStream_t st) {
    using C = Cfg<EPI>;
    // k-steps per weight copy: consecutive k-steps are contiguous when the
    // array holds exactly this kernel's projections; up to 18 KB per copy
    a.wchunk = 1;
    if (a.wstride == C::NP)
        for (int ch = 4; ch > 1; ch >>= 1)
            if (a.n_kt % ch == 0 && ch * C::W_STAGE <= C::W_BYTES / 6) {
                a.wchunk = ch;
                break;
            }
    const int smem = C::SMEM;
    auto kern = a.trace ? k_gemm<EPI, true> : k_gemm<EPI, false>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    kern<<<num_sms, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st) {
    if (a.bn > kBN || a.bn % kSegAlign || (epi == kEpiSwiglu && (a.wstride < 2 || !a.x_rows || !a.src)))
        return cudaErrorInvalidValue;
    switch (epi) {
        case kEpiSwiglu: return launch_t<kEpiSwiglu>(a, num_sms, st);
        case kEpiBf16: return launch_t<kEpiBf16>(a, num_sms, st);
        case kEpiF32: return launch_t<kEpiF32>(a, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace obs
