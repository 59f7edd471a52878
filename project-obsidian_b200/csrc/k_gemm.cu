// k_gemm.cu -- prefill expert FFN: grouped 4-bit dequant GEMM on tcgen05.
//
// Replaces the reference's per-expert matmul_dequant_4bit dispatches
// (shaders/matmul_dequant_4bit.metal:21-66; host src/forward.rs:313-321,
// per-expert calls :219-222) and the ew_swiglu between them (ops.metal:18-22).
//
// One persistent CTA per SM walks work items (token tile of <= 64 rows, weight
// row tile of 128 rows).  An item's reduction dimension is walked in pipeline
// steps of two k-groups (K = 128): every role synchronises once per step, so
// the fixed cost of its barrier waits, fences and TMEM-store waits (each a few
// hundred cycles on a busy SM) is spread over twice the work of one group.
// Twenty-four warps in five roles:
//   warp 0      weight producer: 1-D bulk async copies of the packed weight
//               blocks of one step (18 KB gate/up, 9 KB down; contiguous by
//               construction of the HBM layout) into a shared-memory ring (W);
//   warp 1      token-tile producer into the B ring: bulk copies (L2
//               evict-last: every row tile re-reads them) of the tile's rows of
//               the tiled activations (128-byte-swizzled K-major 8-row atoms):
//               for gate/up the routed input rows the dispatch permuted, for
//               down the H rows of the gate/up epilogue;
//   warps 2-3   MMA issuers (the warp runs converged, one elected lane issues):
//               tcgen05.mma kind::f16 with A in TMEM and B in shared memory,
//               M = 128 weight rows, N = token rows, K = 16, fp32 accumulators
//               in TMEM.  Issuer 0 owns the gate chain (or the even k-slices),
//               issuer 1 the up chain (odd k-slices); one thread issues an MMA
//               only every ~50 cycles, two keep the tensor pipe busy.  Two
//               accumulator buffers let the epilogue overlap the next item; a
//               step's A and B stages are free once both issuers' commits of
//               that step have arrived;
//   warps 4-19  dequantise a W stage (released as soon as it is read) straight
//               into tensor memory: two codes per bf16x2 register,
//               q = (0x4300 | n) - 128, w = fma.rn.bf16x2(q, s, b) (the correctly
//               rounded bf16 of q*s + b), written with tcgen05.st into an A stage
//               of TMEM (one weight row per TMEM lane); each warp owns the TMEM
//               lane quarter it may access and is software-pipelined (the next
//               step's packed words are read while its TMEM store drains);
//   warps 20-23 epilogue: tcgen05.ld, SwiGLU (or plain), results staged in
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
constexpr int kKS = 2;   // k-groups (K = 64 each) per pipeline step
constexpr int kDqWarps = 16, kEpWarps = 4;
// twenty-four warps, six per SM sub-partition (registers are allocated per
// sub-partition: 6 x 32 x 80 fit its 16384); four dequant warps per
// sub-partition hide each other's barrier and TMEM-store latency
constexpr int kWarpW = 0, kWarpB = 1, kWarpMma = 2, kMmaWarps = 2, kWarpDq = kWarpMma + kMmaWarps,
              kWarpEp = kWarpDq + kDqWarps;
constexpr int kThreads = 32 * (kWarpEp + kEpWarps);  // 768
constexpr int kEpThreads = 32 * kEpWarps;

template <int EPI>
struct Cfg {
    static constexpr int NP = EPI == kEpiSwiglu ? 2 : 1;  // projections per tile (gate, up)
    static constexpr int KB = NP * kBlockBytes;           // packed weights of one k-group
    static constexpr int W_STEP = kKS * KB;               // ... of one pipeline step
    static constexpr int W_BYTES = 6 * 2 * 2 * kBlockBytes;  // W ring: 110592 bytes
    static constexpr int SW = W_BYTES / W_STEP;            // 6 (gate/up) or 12 stages
    static constexpr int B_GROUP = kBN * 128;             // one k-group of the token tile (SW128 K-major)
    static constexpr int B_STAGE = kKS * B_GROUP;
    static constexpr int SB = 4;                          // B stages (the gather's L2 latency)
    // accumulators per buffer: gate + up, or (single projection) even + odd k-slices,
    // so the two issuers always target independent accumulators
    static constexpr int ACC_COLS = 2 * kBN;              // one accumulator buffer (fp32 columns)
    static constexpr int A_COLS = NP * kKS * 32;          // one A stage: 64 bf16 per row and group = 32 columns
    static constexpr int A_TMEM = 2 * ACC_COLS;           // first A stage column
    static constexpr int TMEM_COLS = 512;
    static constexpr int SA = (TMEM_COLS - A_TMEM) / A_COLS;  // 2 (gate/up) or 4 A stages
    static constexpr int STG = kBN * 256;                 // epilogue staging: 64 rows x 128 features bf16
    static constexpr int B_OFF = 0;                       // 1024-aligned tiles first
    static constexpr int STG_OFF = B_OFF + SB * B_STAGE;
    static constexpr int W_OFF = STG_OFF + 2 * STG;
    static constexpr int BAR_OFF = (W_OFF + W_BYTES + 7) / 8 * 8;
    static constexpr int N_BARS = 2 * SW + 2 * SB + SA + 4;
    static constexpr int SMEM = BAR_OFF + N_BARS * 8 + 32 + 1024;  // + alignment slack
};
static_assert(Cfg<kEpiSwiglu>::SMEM <= 232448, "smem");
static_assert(Cfg<kEpiBf16>::SMEM <= 232448, "smem");
static_assert(Cfg<kEpiSwiglu>::SA >= 2 && Cfg<kEpiBf16>::SA >= 2, "tmem");

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
    pdl_begin();
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
    auto accfull = [&](int b) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + C::SA + b); };
    auto accempty = [&](int b) { return bar_base + 8 * (2 * C::SW + 2 * C::SB + C::SA + 2 + b); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        // a W stage and an A stage are read / written by one group of eight dequant warps
        for (int s = 0; s < C::SW; ++s) mbar_init(full_w(s), 1), mbar_init(empty_w(s), kDqWarps / 2);
        // "step done" (frees its B stage and its A stage) and "accumulator full"
        // complete on one commit from each issuer
        for (int s = 0; s < C::SB; ++s) mbar_init(full_b(s), 1), mbar_init(empty_b(s), kMmaWarps);
        for (int s = 0; s < C::SA; ++s) mbar_init(aready(s), kDqWarps / 2);
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
    const int KS = a.n_kt / kKS;  // pipeline steps per item
    // consecutive k-groups of one (expert, row tile) are contiguous when the
    // array holds exactly this kernel's projections: one copy per step
    const bool w_contig = a.wstride == C::NP;

    if (warp == kWarpW) {
        // ---------------------------------------------- weight producer (bulk)
        const uint64_t pol = policy_evict_first();
        int s = 0, ph = 0, issued = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            const uint8_t* wsrc =
                a.wblocks + (((size_t)tl.x * a.n_rt + rt) * a.n_kt * a.wstride + a.woff) * kBlockBytes;
            for (int ks = 0; ks < KS; ++ks) {
                if (!wait_all(empty_w(s), ph ^ 1, abort_flag)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(full_w(s), C::W_STEP);
                    const uint8_t* src = wsrc + (size_t)ks * kKS * a.wstride * kBlockBytes;
                    const uint32_t dst = sbase + C::W_OFF + s * C::W_STEP;
                    if (w_contig) {
                        bulk_g2s_hint(dst, src, C::W_STEP, full_w(s), pol);
                    } else {
#pragma unroll
                        for (int g = 0; g < kKS; ++g)
                            bulk_g2s_hint(dst + g * C::KB, src + (size_t)g * a.wstride * kBlockBytes, C::KB, full_w(s),
                                          pol);
                    }
                }
                __syncwarp();
                if (lane == 0) trace_at<TRACE>(a, kTrWIssue, issued);
                ++issued;
                if (++s == C::SW) s = 0, ph ^= 1;
            }
        }
        if (*abort_flag && lane == 0) drain_ring(full_w(0), C::SW, issued);
        __syncwarp();
    } else if (warp == kWarpB) {
        // ----------------------------------------------- token-tile producer
        const uint64_t pol = policy_evict_last();
        int s = 0, ph = 0, issued = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(a.act) + (size_t)(tl.y >> 3) * 1024;
            const uint32_t bbytes = (uint32_t)tl.z * 128u;
            for (int ks = 0; ks < KS; ++ks) {
                if (!wait_all(empty_b(s), ph ^ 1, abort_flag)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(full_b(s), kKS * bbytes);
#pragma unroll
                    for (int g = 0; g < kKS; ++g)
                        bulk_g2s_hint(sbase + C::B_OFF + s * C::B_STAGE + g * C::B_GROUP,
                                      xsrc + (size_t)(ks * kKS + g) * a.atoms * 1024, bbytes, full_b(s), pol);
                }
                __syncwarp();
                if (lane == 0) trace_at<TRACE>(a, kTrBSignal, issued);
                ++issued;
                if (++s == C::SB) s = 0, ph ^= 1;
            }
        }
        if (*abort_flag && lane == 0) drain_ring(full_b(0), C::SB, issued);
        __syncwarp();
    } else if (warp < kWarpMma + kMmaWarps) {
        // --------------------------------------------------------- MMA issuers
        // issuer mi: gate/up -> projection mi (its own accumulator chain, 8
        // k-slices per step); single projection -> k-slices mi, mi+2, mi+4, mi+6
        // of the step into accumulator mi (even/odd, summed by the epilogue).
        // The whole warp runs the loop (waits, descriptor arithmetic) and one
        // elected lane issues: a loop run by lane 0 alone issues far slower.
        const int mi = warp - kWarpMma;
        int sa = 0, pha = 0, sb = 0, phb = 0, it = 0, step = 0;
        const uint32_t a_tmem0 = tmem + C::A_TMEM + (C::NP == 2 ? mi * kKS * 32 : 0);
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
            for (int ks = 0; ks < KS; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(aready(sa), pha, abort_flag) &&
                                                  mbar_wait(full_b(sb), phb, abort_flag))) {
                    ok = false;
                    break;
                }
                if (tr) trace_at<TRACE>(a, kTrMmaStart, step);
                tc_fence_after();
                if (tr) trace_at<TRACE>(a, kTrMmaFenced, step);
                // descriptors: plain adds on precomputed bases (the start address field
                // advances 16 bytes per unit; stages stay below 256 KB).  k-slice kk of the
                // step: A columns kk*8 of this issuer's part, B group kk/4, 32 bytes per slice.
                const uint32_t abase = a_tmem0 + sa * C::A_COLS;
                const uint64_t bdesc = b_desc0 + (uint64_t)(sb * (C::B_STAGE >> 4));
                if (elect_one()) {
                    if constexpr (C::NP == 2) {
#pragma unroll
                        for (int kk = 0; kk < 4 * kKS; ++kk)
                            tc_mma_f16_ts(dbase, abase + kk * 8, bdesc + (kk >> 2) * (C::B_GROUP >> 4) + 2 * (kk & 3),
                                          idesc, (ks | kk) != 0 ? 1u : 0u);
                    } else {
#pragma unroll
                        for (int k2 = 0; k2 < 4 * kKS; k2 += 2) {
                            const int kk = k2 + mi;
                            tc_mma_f16_ts(dbase, abase + kk * 8, bdesc + (kk >> 2) * (C::B_GROUP >> 4) + 2 * (kk & 3),
                                          idesc, (ks | k2) != 0 ? 1u : 0u);
                        }
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
        // Two groups of eight warps take alternate steps (group gi the steps
        // i = gi mod 2), so each warp's chain of waits, TMEM stores and loads
        // spans two step periods.  Warp w of a group: TMEM lane quarter q (rows
        // 32q..32q+31) and part p = w >> 2 of the step: gate/up -> projection p
        // (its 8 words in each of the step's two k-groups), single projection ->
        // k-group p (its 8 words).
        constexpr int NGW = C::NP == 2 ? kKS : 1;  // k-groups per warp and step
        const int dw = warp - kWarpDq;             // 0..15
        const int gi = dw >> 3;                    // step parity of this group
        const int q = warp & 3;                    // TMEM lane quarter this warp may write
        const int r = q * 32 + lane;               // weight row of the tile = TMEM lane
        const int part = (dw >> 2) & 1;
        // packed block of (first k-group, projection) in a W stage
        const int boff = C::NP == 2 ? part * kBlockBytes : part * C::KB;
        // A stage columns: [projection][k-group][32] (gate/up) or [k-group][32]
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + C::A_TMEM + part * NGW * 32;
        const bool tr = TRACE && dw == 0 && lane == 0;
        const int my_items = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int total = my_items * KS;
        uint32_t ws[8 * NGW], s2v[NGW], b2v[NGW];
        // read the packed words (and the row's scales and biases) of step i, release the W stage
        auto load_w = [&](int i) -> bool {
            const int ls = i % C::SW;
            if (!wait_all(full_w(ls), (i / C::SW) & 1, abort_flag)) return false;
            if (tr) trace_at<TRACE>(a, kTrDqStart, i);
#pragma unroll
            for (int g = 0; g < NGW; ++g) {
                const uint8_t* blk = smem + C::W_OFF + ls * C::W_STEP + boff + g * C::KB;
                const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
                const uint32_t sv = sb[r], bv = sb[kRowTile + r];
                s2v[g] = sv | (sv << 16);
                b2v[g] = bv | (bv << 16);
                // word w of row r lives in plane w/4 of the block
#pragma unroll
                for (int pl = 0; pl < 2; ++pl) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(blk + pl * 2048 + r * 16);
                    ws[8 * g + 4 * pl] = w0.x, ws[8 * g + 4 * pl + 1] = w0.y;
                    ws[8 * g + 4 * pl + 2] = w0.z, ws[8 * g + 4 * pl + 3] = w0.w;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_w(ls));  // packed blocks consumed: recycle early
            return true;
        };
        bool ok = gi >= total || load_w(gi);
        for (int step = gi; step < total && ok; step += 2) {
            const int sa = step % C::SA;
            const uint32_t at = trow + sa * C::A_COLS;
#pragma unroll
            for (int g = 0; g < NGW; ++g) {
                uint32_t v[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) dequant_word(ws[8 * g + c], s2v[g], b2v[g], &v[4 * c]);
                if (g == 0) {
                    // A stage sa was last read by the MMAs of step (step - SA)
                    const int prev = step - C::SA;
                    if (prev >= 0 && !wait_all(empty_b(prev % C::SB), (prev / C::SB) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                tmem_st32(at + g * 32, v);
            }
            if (!ok) break;
            if (tr) trace_at<TRACE>(a, kTrDqStored, step);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aready(sa));
            if (tr) trace_at<TRACE>(a, kTrDqDone, step);
            // the group's next step is two steps away: its load is off the critical loop
            if (step + 2 < total && !load_w(step + 2)) ok = false;
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
                            const float hv = silu_mul(gv, u[jj]);
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
                if constexpr (EPI == kEpiSwiglu) {
                    fence_proxy_async_smem();  // staging written by threads -> read by the bulk copy
                    named_bar_sync(1, kEpThreads);
                    if (et == 0) {
                        // two 64-feature planes of the tiled H, each one contiguous run of the tile's atoms
                        uint8_t* hb = reinterpret_cast<uint8_t*>(a.out);
#pragma unroll
                        for (int pln = 0; pln < 2; ++pln)
                            bulk_s2g(hb + ((size_t)(rt * 2 + pln) * a.out_atoms + (tl.y >> 3)) * 1024,
                                     sbase + C::STG_OFF + buf * C::STG + pln * (kBN * 128), (uint32_t)tl.z * 128u);
                        bulk_commit();
                        trace_at<TRACE>(a, kTrEpDone, it);
                    }
                } else {
                    // row-major Y: 256 bytes per token row at a 2*out_ld stride; all
                    // epilogue threads copy the staged rows out in 16-byte pieces
                    named_bar_sync(1, kEpThreads);
                    uint8_t* yb = reinterpret_cast<uint8_t*>(a.out) + ((size_t)tl.y * a.out_ld + rt * kRowTile) * 2;
                    const int nstore = min(tl.z, a.row_limit - tl.y);
                    for (int i = et; i < nstore * 16; i += kEpThreads) {
                        const int j = i >> 4, c = i & 15;
                        *reinterpret_cast<uint4*>(yb + (size_t)j * a.out_ld * 2 + c * 16) =
                            *reinterpret_cast<const uint4*>(stg + j * 256 + c * 16);
                    }
                    if (et == 0) trace_at<TRACE>(a, kTrEpDone, it);
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
static cudaError_t launch_t(const GemmArgs& a, int num_sms, cudaStream_t st) {
    const int smem = Cfg<EPI>::SMEM;
    auto kern = a.trace ? k_gemm<EPI, true> : k_gemm<EPI, false>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    {
        const cudaError_t le_ = launch_pdl(kern, dim3(num_sms), dim3(kThreads), smem, st, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st) {
    if (a.bn > kBN || a.bn % kSegAlign || a.n_kt % kKS || !a.act || (epi == kEpiSwiglu && a.wstride < 2))
        return cudaErrorInvalidValue;
    switch (epi) {
        case kEpiSwiglu: return launch_t<kEpiSwiglu>(a, num_sms, st);
        case kEpiBf16: return launch_t<kEpiBf16>(a, num_sms, st);
        case kEpiF32: return launch_t<kEpiF32>(a, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace obs
