// k_gemm.cu -- prefill expert FFN: grouped 4-bit dequant GEMM on tcgen05.
//
// Replaces the reference's per-expert matmul_dequant_4bit dispatches
// (shaders/matmul_dequant_4bit.metal:21-66; host src/forward.rs:313-321,
// per-expert calls :219-222) and the ew_swiglu between them (ops.metal:18-22).
//
// One persistent CTA per SM walks work items (token tile of <= BN rows, weight
// row tile).  The MMA is M = 128 weight rows x N = the tile's token rows, so a
// dequantised weight row feeds up to BN tokens.  The template has two forms:
// BN = 64, the one launched (the two accumulator buffers of 64 columns leave TMEM
// room for six A stages, so the dequant warps run three pairs of steps ahead of
// the MMAs), and BN = 128 (halves the 4-bit -> bf16 unpack per token), withdrawn
// after an unexplained device fault on workloads with many 65-127-row tiles.  To fit the SwiGLU
// pair into one accumulator, the gate/up weight array is "paired": each 128-row
// block holds 64 gate rows and the matching 64 up rows, interleaved by TMEM lane
// quarter (rows 32q + i: gate feature 16q + i for i < 16, up feature 16q + i - 16
// for i >= 16), so one MMA chain yields gate and up of 64 features and the
// epilogue pairs them with one shuffle across lanes i and i + 16.
//
// The reduction dimension is walked in MMA steps of two k-groups (K = 128).
// Twenty-four warps:
//   warp 0      weight producer: one 1-D bulk async copy of four k-groups
//               (18 KB, contiguous by construction of the HBM layout) per W
//               stage (= two MMA steps);
//   warps 1, 3  token-tile producers: bulk copies (L2 evict-last: every row
//               tile re-reads them) of the tile's rows of the tiled activations
//               (128-byte-swizzled K-major 8-row atoms): for gate/up the routed
//               input rows the dispatch permuted, for down the H rows of the
//               gate/up epilogue.  Warp 1 copies the first k-group of each MMA
//               step, warp 3 the second: one thread takes ~200 ns to issue an
//               8 KB bulk copy, so a single producer issuing both (~400 ns per
//               step) held the MMAs back at large batches;
//   warp 2      MMA issuer (the warp runs converged, one elected lane issues):
//               tcgen05.mma kind::f16, A in TMEM, B in shared memory, K = 16,
//               eight per step, fp32 accumulators in TMEM.  One thread issues an
//               MMA every ~40 cycles and each mbarrier wait costs it more than a
//               hundred, so it waits once per pair of steps (16 MMAs), on a
//               barrier that says both steps' A and B stages are ready, and
//               frees both with one commit;
//   warps 4-19  four dequant quads (one warp per lane quarter); quad j owns the
//               MMA steps j mod 4 (A and B stage: step mod SA), so each warp has
//               four step periods for its share: read the packed words of its 32 rows x
//               two k-groups from the W stage, unpack two codes per bf16x2
//               register, w = fma.rn.bf16x2(n as a subnormal, s * 2^133, b)
//               (the correctly rounded bf16 of n*s + b; scales outside that
//               form's range take q = (0x4300 | n) - 128 first), write them with
//               tcgen05.st into the A stage (one weight row per TMEM lane), wait
//               for the step's token tile to land, and arrive on the pair's
//               ready barrier;
//   warps 20-23 epilogue: tcgen05.ld, SwiGLU (or plain), results staged in
//               shared memory in the global layout and written back with bulk
//               copies or 16-byte stores (fp32 debug output: direct stores).
// Keeping A out of shared memory leaves shared-memory bandwidth to the weight
// and token streams.  The packed words hold their codes in the nibble order
// (c0,c2,c4,c6,c1,c3,c5,c7) (set by the loader), so (w >> 4j) & 0x000F000F is
// the bf16x2 pair of columns (2j, 2j+1).
// Every mbarrier wait is bounded; a CTA that gives up records kDevTimeout,
// drains its outstanding copies (bounded), frees its TMEM and returns.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kKS = 2;     // k-groups (K = 64 each) per MMA step
constexpr int kWK = 4;     // k-groups per weight copy (one W stage = two MMA steps)
constexpr int kQuads = 4;  // dequant quads; quad j owns MMA steps j mod 4
constexpr int kDqWarps = 4 * kQuads, kEpWarps = 4;
constexpr int kWarpW = 0, kWarpB = 1, kWarpMma = 2, kWarpB2 = 3, kWarpDq = 4, kWarpEp = kWarpDq + kDqWarps;
constexpr int kThreads = 32 * (kWarpEp + kEpWarps);  // 768
constexpr int kEpThreads = 32 * kEpWarps;

// BN = token rows per tile (tcgen05 N).  TMEM holds two accumulator buffers of BN
// fp32 columns and the A stages (64 columns each) in the rest: four stages (two
// pair slots) at BN = 128, six (three pair slots) at BN = 64, so with small tiles
// the dequant warps can run one more pair ahead of the MMAs.  Step s uses A and
// B stage s % SA; pair slot p covers stages 2p, 2p+1.
template <int BN>
struct Cfg {
    static constexpr int NPS = BN >= 128 ? 2 : 3;      // pair slots
    static constexpr int SA = 2 * NPS, SB = SA;        // A stages (TMEM), B stages (shared memory)
    static constexpr int W_STAGE = kWK * kBlockBytes;  // 18432
    static constexpr int SW = BN >= 128 ? 3 : 5;       // W stages (two MMA steps each)
    static constexpr int B_GROUP = BN * 128;           // one k-group of the token tile (SW128 K-major)
    static constexpr int B_STAGE = kKS * B_GROUP;
    static constexpr int ACC_COLS = BN;                // one accumulator buffer (fp32 columns)
    static constexpr int A_COLS = kKS * 32;            // one A stage: 64 bf16 per row and k-group = 32 columns
    static constexpr int A_TMEM = 2 * ACC_COLS;        // first A stage column
    static constexpr int TMEM_COLS = 512;
    static constexpr int STG = BN * 256;               // epilogue staging: BN rows x 128 features bf16
    static constexpr int B_OFF = 0;                    // 1024-aligned tiles first
    static constexpr int STG_OFF = B_OFF + SB * B_STAGE;
    static constexpr int W_OFF = STG_OFF + STG;
    static constexpr int BAR_OFF = W_OFF + SW * W_STAGE;
    static constexpr int N_BARS = 2 * SW + SB + 2 * NPS + 4 + 1;
    static constexpr int SMEM = BAR_OFF + N_BARS * 8 + 32 + 1024;  // + alignment slack
    static_assert(SMEM <= 232448, "smem");
    static_assert(A_TMEM + SA * A_COLS <= TMEM_COLS, "tmem");
};
static_assert(kWK == 2 * kKS, "a W stage holds two MMA steps");

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

// The same in one instruction per pair: the masked code n, read as a bf16 bit
// pattern, is the subnormal n * 2^-133, and s2 carries the scale times 2^133
// (its exponent field raised by 133, exact), so the product is exactly n * s and
// fma.rn gives round(n * s + b), bit for bit the value above.  Valid for scales
// with exponent field 1..121 (2^-126 <= |s| < 2^-5); the caller falls back to
// dequant_word for any other group.
__device__ __forceinline__ void dequant_word_sub(uint32_t w, uint32_t s2x, uint32_t b2, uint32_t* out) {
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = bf2_fma((w >> (4 * j)) & 0x000F000Fu, s2x, b2);
}
constexpr uint32_t kSubExpShift = 133u << 7;  // + 133 in a bf16 exponent field
__device__ __forceinline__ bool sub_form_ok(uint32_t s_bits) {
    const uint32_t ex = (s_bits >> 7) & 0xFFu;
    return ex >= 1u && ex <= 121u;
}

// which wait timed out (recorded in the context's second error word)
enum WaitCode : int { kWtEmptyW = 11, kWtSfreeB, kWtAccEmpty, kWtAReady, kWtFullW, kWtSfreeA, kWtFullB, kWtAccFull };

__device__ __forceinline__ bool wait_all(uint32_t bar, uint32_t parity, volatile int* abort, int code,
                                         uint64_t limit_ns) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, code, limit_ns));
}

// After giving up, a producer waits (bounded) until the newest copy it issued
// into each stage of its ring has landed, so no copy targets freed memory.
__device__ __forceinline__ void drain_ring(uint32_t bar0, int stages, int issued, uint64_t limit_ns) {
    for (int st = 0; st < stages && st < issued; ++st) {
        const int last = st + (issued - 1 - st) / stages * stages;
        const uint32_t par = (last / stages) & 1;
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(bar0 + 8 * st, par) && global_ns() - t0 < limit_ns) {
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

template <int EPI, int BN, bool TRACE>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(GemmArgs a) {
    pdl_begin();
    using C = Cfg<BN>;
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
    // pair slot ps = (step / 2) % NPS covers the A and B stages 2ps, 2ps + 1
    constexpr int PB = 2 * C::SW + C::SB;
    auto aready = [&](int ps) { return bar_base + 8 * (PB + ps); };
    auto sfree = [&](int ps) { return bar_base + 8 * (PB + C::NPS + ps); };
    auto accfull = [&](int b) { return bar_base + 8 * (PB + 2 * C::NPS + b); };
    auto accempty = [&](int b) { return bar_base + 8 * (PB + 2 * C::NPS + 2 + b); };
    const uint32_t mma_done = bar_base + 8 * (PB + 2 * C::NPS + 4);  // the issuer's last commit

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        // a W stage is read by the two quads of its two MMA steps (four warps each)
        for (int s = 0; s < C::SW; ++s) mbar_init(full_w(s), 1), mbar_init(empty_w(s), 8);
        // a pair of steps is ready when its two quads (eight warps) have written A and
        // seen B land; one issuer commit frees its A and B stages
        for (int s = 0; s < C::SB; ++s) mbar_init(full_b(s), kKS);  // one arrival per k-group producer
        for (int ps = 0; ps < C::NPS; ++ps) mbar_init(aready(ps), 8), mbar_init(sfree(ps), 1);
        for (int b = 0; b < 2; ++b) mbar_init(accfull(b), 1), mbar_init(accempty(b), kEpThreads);
        mbar_init(mma_done, 1);
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
    const int n_tiles = *a.n_tiles;
    // (each tile holds >= 16 rows, so a count above atoms / 2 is corrupt)
    const bool count_ok = n_tiles >= 0 && n_tiles <= a.atoms / 2 && n_tiles <= a.max_tiles;
    const int n_items = count_ok ? n_tiles * a.n_rt : 0;
    const int KS = a.n_kt / kKS;  // MMA steps per item (even: n_kt is a multiple of 4)
    // Every role walks the same items, so a tile outside the buffers (a corrupt
    // tile list) is refused up front by the whole CTA: error recorded, no work.
    {
        bool bad = !count_ok;
        for (int item = blockIdx.x + tid * gridDim.x; item < n_items; item += blockDim.x * gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            bad |= tl.x < 0 || tl.x >= a.n_experts || tl.y < 0 || (tl.y & 15) || tl.z < kSegAlign || tl.z > a.bn ||
                   (tl.z & 15) || tl.y + tl.z > a.atoms * 8;
        }
        if (__syncthreads_or(bad)) {
            if (tid == 0) atomicExch(a.err, kDevBadTile);
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (warp == kWarpMma) tmem_dealloc(tmem, C::TMEM_COLS);
            return;
        }
    }

    if (warp == kWarpW) {
        // ---------------------------------------------- weight producer (bulk)
        const uint64_t pol = policy_evict_first();
        int s = 0, ph = 0, issued = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            const uint8_t* wsrc = a.wblocks + ((size_t)tl.x * a.n_rt + rt) * a.n_kt * kBlockBytes;
            for (int w = 0; w < a.n_kt / kWK; ++w) {
                if (!wait_all(empty_w(s), ph ^ 1, abort_flag, kWtEmptyW, a.wait_ns)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(full_w(s), C::W_STAGE);
                    bulk_g2s_hint(sbase + C::W_OFF + s * C::W_STAGE, wsrc + (size_t)w * C::W_STAGE, C::W_STAGE,
                                  full_w(s), pol);
                }
                __syncwarp();
                if (lane == 0) trace_at<TRACE>(a, kTrWIssue, issued);
                ++issued;
                if (++s == C::SW) s = 0, ph ^= 1;
            }
        }
        if (*abort_flag && lane == 0) drain_ring(full_w(0), C::SW, issued, a.wait_ns);
        __syncwarp();
    } else if (warp == kWarpB || warp == kWarpB2) {
        // ------------------------------------- token-tile producers (k-group g)
        const int g = warp == kWarpB ? 0 : 1;
        static_assert(kKS == 2, "one producer warp per k-group of an MMA step");
        const uint64_t pol = policy_evict_last();
        int s = 0, ph = 0, issued = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int4 tl = a.tiles[item / a.n_rt];
            const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(a.act) + (size_t)(tl.y >> 3) * 1024;
            const uint32_t bbytes = (uint32_t)tl.z * 128u;
            for (int ks = 0; ks < KS; ++ks) {
                if (!wait_all(sfree(s >> 1), ph ^ 1, abort_flag, kWtSfreeB, a.wait_ns)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(full_b(s), bbytes);
                    bulk_g2s_hint(sbase + C::B_OFF + s * C::B_STAGE + g * C::B_GROUP,
                                  xsrc + (size_t)(ks * kKS + g) * a.atoms * 1024, bbytes, full_b(s), pol);
                }
                __syncwarp();
                if (g == 0 && lane == 0) trace_at<TRACE>(a, kTrBSignal, issued);
                ++issued;
                if (++s == C::SB) s = 0, ph ^= 1;
            }
        }
        // (a phase the other producer never fed ends the drain at its time limit)
        if (*abort_flag && lane == 0) drain_ring(full_b(0), C::SB, issued, a.wait_ns);
        __syncwarp();
    } else if (warp == kWarpMma) {
        // ---------------------------------------------------------- MMA issuer
        // The whole warp runs the loop (waits, descriptor arithmetic) and one
        // elected lane issues: a loop run by lane 0 alone issues far slower.
        // One wait, one fence and one commit per pair of steps (16 MMAs): every
        // mbarrier wait costs the issuing thread more than a hundred cycles.
        int pair = 0, it = 0;
        const uint64_t b_desc0 = sw128_desc(sbase + C::B_OFF);
        const bool tr = TRACE && lane == 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++it) {
            const int4 tl = a.tiles[item / a.n_rt];
            const uint32_t idesc = idesc_bf16(128, tl.z);
            const int buf = it & 1;
            if (!wait_all(accempty(buf), ((it >> 1) & 1) ^ 1, abort_flag, kWtAccEmpty, a.wait_ns)) break;
            tc_fence_after();
            const uint32_t dbase = tmem + buf * C::ACC_COLS;
            bool ok = true;
            for (int pi = 0; pi < KS / 2; ++pi, ++pair) {
                const int ps = pair % C::NPS;
                if (!wait_all(aready(ps), (pair / C::NPS) & 1, abort_flag, kWtAReady, a.wait_ns)) {
                    ok = false;
                    break;
                }
                if (tr) trace_at<TRACE>(a, kTrMmaStart, pair);
                tc_fence_after();
                if (tr) trace_at<TRACE>(a, kTrMmaFenced, pair);
                // descriptors: plain adds on precomputed bases (the start address field
                // advances 16 bytes per unit; stages stay below 256 KB).  k-slice kk of
                // step stage sa: A columns kk*8, B group kk/4, 32 bytes per slice.
                if (elect_one()) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int sa = 2 * ps + h;
                        const uint32_t abase = tmem + C::A_TMEM + sa * C::A_COLS;
                        const uint64_t bdesc = b_desc0 + (uint64_t)(sa * (C::B_STAGE >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4 * kKS; ++kk)
                            tc_mma_f16_ts(dbase, abase + kk * 8, bdesc + (kk >> 2) * (C::B_GROUP >> 4) + 2 * (kk & 3),
                                          idesc, (pi | h | kk) != 0 ? 1u : 0u);
                    }
                    tc_commit(sfree(ps));  // the pair's MMAs are done: its A and B stages are free
                }
                __syncwarp();
                if (tr) trace_at<TRACE>(a, kTrMmaIssued, pair);
            }
            if (!ok) break;
            if (elect_one()) tc_commit(accfull(buf));
            __syncwarp();
        }
        // Every MMA this thread issued has finished before the CTA frees its tensor
        // memory, also when a role gave up mid-item (bounded; no abort check).
        if (elect_one()) tc_commit(mma_done);
        __syncwarp();
        {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(mma_done, 0) && global_ns() - t0 < a.wait_ns) {
            }
        }
        __syncwarp();
    } else if (warp >= kWarpDq && warp < kWarpEp) {
        // ------------------------------------------------------------ dequant
        // Quad j (warps 4j+4 .. 4j+7) owns the MMA steps i = j mod 4; step i writes
        // A stage i % SA and reads half (i & 1) of W stage i / 2: k-groups 2(i&1), 2(i&1)+1.
        const int dw = warp - kWarpDq;  // 0..15
        const int j = dw >> 2;          // quad
        const int q = warp & 3;         // TMEM lane quarter this warp may write
        const int r = q * 32 + lane;    // weight row of the tile = TMEM lane
        const uint32_t at0 = tmem + ((uint32_t)(q * 32) << 16) + C::A_TMEM;
        const bool tr = TRACE && dw == 0 && lane == 0;
        const bool trq = TRACE && dw > 0 && dw < 4 && lane == 0;  // the other quarters of quad 0
        const int my_items = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int total = my_items * KS;
        uint32_t ws[8 * kKS], s2v[kKS], b2v[kKS];
        bool subf[kKS];  // this row's group takes the subnormal form (s2v then holds s * 2^133)
        // read the packed words (and the row's scales and biases) of step i, release its half of the W stage
        auto load_w = [&](int i) -> bool {
            const int wi = i >> 1, ls = wi % C::SW;
            if (!wait_all(full_w(ls), (wi / C::SW) & 1, abort_flag, kWtFullW, a.wait_ns)) return false;
            if (tr) trace_at<TRACE>(a, kTrDqStart, i);
#pragma unroll
            for (int g = 0; g < kKS; ++g) {
                const uint8_t* blk = smem + C::W_OFF + ls * C::W_STAGE + ((i & 1) * kKS + g) * kBlockBytes;
                const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
                const uint32_t sv = sb[r], bv = sb[kRowTile + r];
                subf[g] = sub_form_ok(sv);
                const uint32_t sx = subf[g] ? sv + kSubExpShift : sv;
                s2v[g] = sx | (sx << 16);
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
        bool ok = j >= total || load_w(j);
        for (int step = j; step < total && ok; step += kQuads) {
            // A stage x was last read by the MMAs of step (step - SA), in pair slot x / 2
            const int x = step % C::SA, use = step / C::SA;
            const uint32_t at = at0 + x * C::A_COLS;
            if (!wait_all(sfree(x >> 1), (use & 1) ^ 1, abort_flag, kWtSfreeA, a.wait_ns)) break;
            tc_fence_after();
            if (tr) trace_at<TRACE>(a, kTrDqAFree, step);
#pragma unroll
            for (int g = 0; g < kKS; ++g) {
                uint32_t v[32];
#pragma unroll
                if (__all_sync(0xffffffffu, subf[g])) {
#pragma unroll
                    for (int c = 0; c < 8; ++c) dequant_word_sub(ws[8 * g + c], s2v[g], b2v[g], &v[4 * c]);
                } else {  // a scale outside the subnormal form's range: per-row choice
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        if (subf[g]) dequant_word_sub(ws[8 * g + c], s2v[g], b2v[g], &v[4 * c]);
                        else dequant_word(ws[8 * g + c], s2v[g], b2v[g], &v[4 * c]);
                    }
                }
                tmem_st32(at + g * 32, v);
            }
            if (tr) trace_at<TRACE>(a, kTrDqStored, step);
            tc_wait_st();
            // the step's token tile (B stage x) must have landed before the pair is ready
            if (!wait_all(full_b(x), use & 1, abort_flag, kWtFullB, a.wait_ns)) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aready(x >> 1));
            if (tr) trace_at<TRACE>(a, kTrDqDone, step);
            if (trq) trace_at<TRACE>(a, kTrDqDoneQ1 + dw - 1, step);
            // the quad's next step is four steps away: its load is off the critical loop
            if (step + kQuads < total && !load_w(step + kQuads)) ok = false;
        }
    } else if (warp >= kWarpEp) {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quarter of this warp
        const int et = tid - 32 * kWarpEp;
        // paired array: lane i < 16 holds gate, i >= 16 up, of feature 16q + (i & 15) of the row tile
        const int hi = (lane >> 4) & 1;
        const int fp = q * 16 + (lane & 15);
        int it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            const int buf = it & 1;
            if (!wait_all(accfull(buf), (it >> 1) & 1, abort_flag, kWtAccFull, a.wait_ns)) break;
            if (et == 0) trace_at<TRACE>(a, kTrEpStart, it);
            tc_fence_after();
            const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + buf * C::ACC_COLS;
            if constexpr (EPI == kEpiF32) {
                const int nstore = min(tl.z, a.row_limit - tl.y);
                const bool mine = !a.paired || hi == a.proj_sel;
                const int f = a.paired ? rt * 64 + fp : rt * kRowTile + q * 32 + lane;
                float* y = reinterpret_cast<float*>(a.out);
                for (int j0 = 0; j0 < tl.z; j0 += 16) {
                    float g[16];
                    tmem_ld16(tq + j0, g);
                    tc_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        if (mine && j0 + jj < nstore) y[(size_t)(tl.y + j0 + jj) * a.out_ld + f] = g[jj];
                }
                tc_fence_before();
                mbar_arrive(accempty(buf));
            } else if constexpr (EPI == kEpiSwiglu) {
                // the previous item's bulk store must have read the staging buffer
                if (et == 0) bulk_wait_read0();
                named_bar_sync(1, kEpThreads);
                uint8_t* stg = smem + C::STG_OFF;
                // lane pair (f, f^1) stores features (f & ~1, +1) as one 4-byte word
                const int odd = lane & 1;
                const int cx = fp >> 3, cb = (fp & 6) << 1;  // 16-byte chunk and byte of the feature pair
                for (int j0 = 0; j0 < tl.z; j0 += 16) {
                    float v[16];
                    tmem_ld16(tq + j0, v);
                    tc_wait_ld();
                    // SwiGLU: lanes i (gate) and i+16 (up) split the 16 tokens, lane i taking
                    // {0-3, 8-11} and lane i+16 {4-7, 12-15} (k-th of each: tk + 4 * hi)
                    float h[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int tk = (k & 3) + ((k >> 2) << 3);
                        const float mine = v[tk + 4 * hi];
                        const float other = __shfl_xor_sync(0xffffffffu, v[tk + 4 * (hi ^ 1)], 16);
                        h[k] = hi ? silu_mul(other, mine) : silu_mul(mine, other);
                    }
                    // tokens a and a + 2 of each half: the even lane of a pair keeps token a, the
                    // odd lane token a + 2, and they swap the other.  One store instruction then
                    // writes tokens a, a+2, a+4, a+6, whose swizzled chunks use disjoint banks.
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const int ka = (p & 1) + ((p >> 1) << 2);  // h index of token a; a + 2 is ka + 2
                        const float keep = odd ? h[ka + 2] : h[ka];
                        const float recv = __shfl_xor_sync(0xffffffffu, odd ? h[ka] : h[ka + 2], 1);
                        const int t = j0 + (ka & 3) + ((ka >> 2) << 3) + 4 * hi + 2 * odd;
                        *reinterpret_cast<uint32_t*>(stg + (t >> 3) * 1024 + (t & 7) * 128 + ((cx ^ (t & 7)) << 4) + cb) =
                            odd ? pack_bf2(recv, keep) : pack_bf2(keep, recv);
                    }
                }
                tc_fence_before();
                mbar_arrive(accempty(buf));  // accumulator drained: the next item may start
                fence_proxy_async_smem();    // staging written by threads -> read by the bulk copy
                named_bar_sync(1, kEpThreads);
                if (et == 0) {
                    // H k-tile rt of the tile's rows: one contiguous run of its atoms
                    uint8_t* hb = reinterpret_cast<uint8_t*>(a.out);
                    bulk_s2g(hb + ((size_t)rt * a.out_atoms + (tl.y >> 3)) * 1024, sbase + C::STG_OFF,
                             (uint32_t)tl.z * 128u);
                    bulk_commit();
                    trace_at<TRACE>(a, kTrEpDone, it);
                }
            } else {
                // row-major Y: 256 bytes per token row at a 2*out_ld stride.  Staging rows
                // are 256 bytes with the 16-byte chunks of odd rows swapped in fours
                // (chunk c at c ^ 4), so the two tokens of one store use disjoint banks.
                named_bar_sync(1, kEpThreads);  // the previous item's rows have been copied out
                uint8_t* stg = smem + C::STG_OFF;
                const int odd = lane & 1;
                const int fb = (q * 32 + (lane & ~1)) * 2;  // byte of the feature pair in a row
                for (int j0 = 0; j0 < tl.z; j0 += 16) {
                    float g[16];
                    tmem_ld16(tq + j0, g);
                    tc_wait_ld();
                    // lane pair (f, f^1): the even lane stores token t, the odd lane token t + 1
#pragma unroll
                    for (int jj = 0; jj < 16; jj += 2) {
                        const float keep = odd ? g[jj + 1] : g[jj];
                        const float recv = __shfl_xor_sync(0xffffffffu, odd ? g[jj] : g[jj + 1], 1);
                        const int t = j0 + jj + odd;
                        *reinterpret_cast<uint32_t*>(stg + t * 256 + (fb ^ (odd << 6))) =
                            odd ? pack_bf2(recv, keep) : pack_bf2(keep, recv);
                    }
                }
                tc_fence_before();
                mbar_arrive(accempty(buf));
                // all epilogue threads copy the staged rows out in 16-byte pieces
                named_bar_sync(1, kEpThreads);
                uint8_t* yb = reinterpret_cast<uint8_t*>(a.out) + ((size_t)tl.y * a.out_ld + rt * kRowTile) * 2;
                const int nstore = min(tl.z, a.row_limit - tl.y);
                if (a.row_ptr) {
                    // expert parallelism: each row goes straight to its destination, for a row
                    // computed for another rank that rank's return buffer over NVLink; a row
                    // without a destination is refused and recorded
                    for (int i = et; i < nstore * 16; i += kEpThreads) {
                        const int jr = i >> 4, c = i & 15;
                        uint8_t* dst = reinterpret_cast<uint8_t*>(a.row_ptr[tl.y + jr]);
                        if (!dst) {
                            if (c == 0) refuse_slot(a.err, kSiteGemmRow, tl.y + jr);
                            continue;
                        }
                        *reinterpret_cast<uint4*>(dst + rt * kRowTile * 2 + c * 16) =
                            *reinterpret_cast<const uint4*>(stg + jr * 256 + ((c ^ ((jr & 1) << 2)) << 4));
                    }
                } else {
                    for (int i = et; i < nstore * 16; i += kEpThreads) {
                        const int jr = i >> 4, c = i & 15;
                        *reinterpret_cast<uint4*>(yb + (size_t)jr * a.out_ld * 2 + c * 16) =
                            *reinterpret_cast<const uint4*>(stg + jr * 256 + ((c ^ ((jr & 1) << 2)) << 4));
                    }
                }
                if (et == 0) trace_at<TRACE>(a, kTrEpDone, it);
            }
        }
        if (et == 0) bulk_wait0();  // results are in global memory before the CTA exits
        if (a.row_ptr) __threadfence_system();  // peer stores ordered before the stamp kernel's
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) tmem_dealloc(tmem, C::TMEM_COLS);
    if (tid == 0 && *abort_flag) {
        atomicExch(a.err + 1, *abort_flag);  // which wait gave up first
        atomicExch(a.err, kDevTimeout);
    }
}

}  // namespace

size_t gemm_smem_bytes(int) { return Cfg<64>::SMEM; }
int gemm_tile_rows() { return 64; }

template <int EPI, int BN>
static cudaError_t launch_t(const GemmArgs& a, int num_sms, cudaStream_t st) {
    const int smem = Cfg<BN>::SMEM;
    auto kern = a.trace ? k_gemm<EPI, BN, true> : k_gemm<EPI, BN, false>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    {
        const cudaError_t le_ = launch_pdl(kern, dim3(num_sms), dim3(kThreads), smem, st, a);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// Only the 64-token form is launched: the 128-token form (Cfg<128>) ended in an
// unexplained device fault on workloads with many 65-127-row tiles and is withdrawn.
cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st) {
    if (a.bn > 64 || a.bn % kSegAlign || a.n_kt % kWK || a.n_kt <= 0 || !a.act || (epi == kEpiSwiglu && !a.paired))
        return cudaErrorInvalidValue;
    switch (epi) {
        case kEpiSwiglu: return launch_t<kEpiSwiglu, 64>(a, num_sms, st);
        case kEpiBf16: return launch_t<kEpiBf16, 64>(a, num_sms, st);
        case kEpiF32: return launch_t<kEpiF32, 64>(a, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace obs
