// k_gemm.cu -- prefill expert FFN: grouped 4-bit dequant GEMM on tcgen05.
//
// Replaces the reference's per-expert matmul_dequant_4bit dispatches
// (shaders/matmul_dequant_4bit.metal:21-66; host src/forward.rs:313-321,
// per-expert calls :219-222) and the ew_swiglu between them (ops.metal:18-22).
//
// One persistent CTA per SM walks work items (token tile, weight row tile):
//   warp 0      producer: 1-D bulk async copies of the packed weight block(s)
//               (4608 B each, contiguous by construction of the HBM layout)
//               and of the token tile (pre-swizzled rows, contiguous per
//               k-tile) into a ring of shared-memory stages;
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, M = 128 weight
//               rows, N = token rows, K = 16, fp32 accumulators in TMEM;
//   warps 2-5   dequantise the packed block into the bf16 A tile in the
//               128-byte-swizzled K-major layout (w = fma(q, s, b), rounded to
//               bf16), then run the epilogue from TMEM (SwiGLU -> tiled H, or
//               a plain bf16 / fp32 store).
// Every mbarrier wait is bounded; a CTA that gives up records kDevTimeout,
// drains its outstanding copies (bounded), frees its TMEM and returns.
#include "obs_internal.cuh"

namespace obs {
namespace {

constexpr int kBN = 128;  // token rows per tile (tcgen05 N <= 128 here)
constexpr int kThreads = 192;

template <int EPI>
struct Cfg {
    static constexpr int NP = EPI == kEpiSwiglu ? 2 : 1;   // projections per tile (gate, up)
    static constexpr int A_BYTES = NP * kRowTile * 128;     // bf16 A tiles, 16 KB each
    static constexpr int B_BYTES = kBN * 128;
    static constexpr int PACK_BYTES = NP * kBlockBytes;
    static constexpr int STAGE = ((A_BYTES + B_BYTES + PACK_BYTES) + 1023) / 1024 * 1024;
    static constexpr int STAGES = EPI == kEpiSwiglu ? 3 : 5;
    static constexpr int TMEM_COLS = NP * kBN;               // 256 or 128
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int SMEM = BAR_OFF + (3 * STAGES + 2) * 8 + 16 + 1024;  // + alignment slack
};

__device__ __forceinline__ uint4 dequant_word(uint32_t w, float sc, float bi) {
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        f[j] = __fmaf_rn(__fsub_rn(__uint_as_float(0x4B000000u | ((w >> (4 * j)) & 0xFu)), 8388608.0f), sc, bi);
    return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(GemmArgs a) {
    using C = Cfg<EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * C::STAGES + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* consumed = reinterpret_cast<volatile int*>(tmem_slot + 2);
    auto full_bar = [&](int s) { return smem_u32(bars + s); };
    auto ready_bar = [&](int s) { return smem_u32(bars + C::STAGES + s); };
    auto empty_bar = [&](int s) { return smem_u32(bars + 2 * C::STAGES + s); };
    const uint32_t accfull_bar = smem_u32(bars + 3 * C::STAGES);
    const uint32_t accempty_bar = smem_u32(bars + 3 * C::STAGES + 1);
    auto a_smem = [&](int s) { return sbase + s * C::STAGE; };
    auto b_smem = [&](int s) { return sbase + s * C::STAGE + C::A_BYTES; };
    auto p_smem = [&](int s) { return smem + s * C::STAGE + C::A_BYTES + C::B_BYTES; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(ready_bar(s), 128);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accfull_bar, 1);
        mbar_init(accempty_bar, 128);
        *abort_flag = 0;
        *consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_items = *a.n_tiles * a.n_rt;
    const int KT = a.n_kt;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
            int s = 0, ph = 0, issued = 0;
            for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
                const int4 tl = a.tiles[item / a.n_rt];
                const int rt = item % a.n_rt;
                const uint8_t* wsrc =
                    a.wblocks + (((size_t)tl.x * a.n_rt + rt) * KT * a.wstride + a.woff) * kBlockBytes;
                const uint32_t bbytes = (uint32_t)tl.z * 128u;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag)) break;
                    mbar_arrive_expect_tx(full_bar(s), C::PACK_BYTES + bbytes);
                    bulk_g2s_hint(smem_u32(p_smem(s)), wsrc + (size_t)kt * a.wstride * kBlockBytes, C::PACK_BYTES,
                                  full_bar(s), pol_w);
                    bulk_g2s_hint(b_smem(s), reinterpret_cast<const uint8_t*>(a.act) +
                                                 ((size_t)kt * a.atoms + (tl.y >> 3)) * 1024,
                                  bbytes, full_bar(s), pol_x);
                    ++issued;
                    if (++s == C::STAGES) s = 0, ph ^= 1;
                }
            }
            // drain: copies still in flight must land before the CTA exits
            if (*abort_flag) {
                for (int i = *consumed; i < issued; ++i) {
                    const int st = i % C::STAGES, par = (i / C::STAGES) & 1;
                    uint64_t t0 = global_ns();
                    while (!mbar_try_wait(full_bar(st), par) && global_ns() - t0 < kWaitLimitNs) {
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int s = 0, ph = 0, it = 0;
            for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++it) {
                const int4 tl = a.tiles[item / a.n_rt];
                const uint32_t idesc = idesc_bf16(128, tl.z);
                if (!mbar_wait(accempty_bar, (it & 1) ^ 1, abort_flag)) break;
                tc_fence_after();
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!mbar_wait(ready_bar(s), ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int p = 0; p < C::NP; ++p)
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc_mma_f16(tmem + p * kBN, sw128_desc(a_smem(s) + p * kRowTile * 128 + kk * 32),
                                       sw128_desc(b_smem(s) + kk * 32), idesc, (kt | kk) != 0);
                    tc_commit(empty_bar(s));
                    if (++s == C::STAGES) s = 0, ph ^= 1;
                }
                if (!ok) break;
                tc_commit(accfull_bar);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------- dequant + epilogue
        const int t = tid - 64;             // weight row of the tile
        const int q = warp & 3;             // TMEM lane quarter of this warp
        const int frow = q * 32 + lane;     // accumulator row read in the epilogue
        int s = 0, ph = 0, it = 0, done = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
            const int4 tl = a.tiles[item / a.n_rt];
            const int rt = item % a.n_rt;
            for (int kt = 0; kt < KT; ++kt) {
                if (!__all_sync(0xffffffffu, mbar_wait(full_bar(s), ph, abort_flag))) { ok = false; break; }
                const uint8_t* pk = p_smem(s);
#pragma unroll
                for (int p = 0; p < C::NP; ++p) {
                    const uint8_t* blk = pk + p * kBlockBytes;
                    const uint4 w0 = *reinterpret_cast<const uint4*>(blk + t * 32);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(blk + t * 32 + 16);
                    const uint16_t* sb = reinterpret_cast<const uint16_t*>(blk + kBlockWords * 4);
                    const float sc = bf2f(sb[t]), bi = bf2f(sb[kRowTile + t]);
                    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    uint8_t* arow = smem + s * C::STAGE + p * kRowTile * 128 + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        *reinterpret_cast<uint4*>(arow + ((c ^ (t & 7)) << 4)) = dequant_word(ws[c], sc, bi);
                }
                fence_proxy_async_smem();
                mbar_arrive(ready_bar(s));
                ++done;
                if (t == 0) *consumed = done;
                if (++s == C::STAGES) s = 0, ph ^= 1;
            }
            if (!ok) break;
            // epilogue
            if (!__all_sync(0xffffffffu, mbar_wait(accfull_bar, it & 1, abort_flag))) { ok = false; break; }
            tc_fence_after();
            const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
            const int feat = rt * kRowTile + frow;
            const int nstore = min(tl.z, a.row_limit - tl.y);
            for (int j0 = 0; j0 < tl.z; j0 += 16) {
                float g[16];
                tmem_ld16(tq + j0, g);
                if constexpr (EPI == kEpiSwiglu) {
                    float u[16];
                    tmem_ld16(tq + kBN + j0, u);
                    tc_wait_ld();
                    uint8_t* hb = reinterpret_cast<uint8_t*>(a.out);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        if (j0 + jj >= nstore) break;
                        const float gv = g[jj];
                        const float hv = (gv / (1.0f + expf(-gv))) * u[jj];  // ops.metal:21
                        *reinterpret_cast<uint16_t*>(hb + tiled_off(tl.y + j0 + jj, feat, a.out_atoms)) = f2bf(hv);
                    }
                } else if constexpr (EPI == kEpiBf16) {
                    tc_wait_ld();
                    uint16_t* y = reinterpret_cast<uint16_t*>(a.out);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        if (j0 + jj < nstore) y[(size_t)(tl.y + j0 + jj) * a.out_ld + feat] = f2bf(g[jj]);
                } else {
                    tc_wait_ld();
                    float* y = reinterpret_cast<float*>(a.out);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        if (j0 + jj < nstore) y[(size_t)(tl.y + j0 + jj) * a.out_ld + feat] = g[jj];
                }
            }
            tc_fence_before();
            mbar_arrive(accempty_bar);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
    if (tid == 0 && *abort_flag) atomicExch(a.err, kDevTimeout);
}

}  // namespace

size_t gemm_smem_bytes(int epi) {
    return epi == kEpiSwiglu ? Cfg<kEpiSwiglu>::SMEM : epi == kEpiBf16 ? Cfg<kEpiBf16>::SMEM : Cfg<kEpiF32>::SMEM;
}

template <int EPI>
static cudaError_t launch_t(const GemmArgs& a, int num_sms, cudaStream_t st) {
    const int smem = Cfg<EPI>::SMEM;
    cudaError_t err = cudaFuncSetAttribute(k_gemm<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    k_gemm<EPI><<<num_sms, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmArgs& a, int epi, int num_sms, cudaStream_t st) {
    if (a.bn > kBN || a.bn % kSegAlign || a.wstride < Cfg<kEpiSwiglu>::NP * (epi == kEpiSwiglu))
        return cudaErrorInvalidValue;
    switch (epi) {
        case kEpiSwiglu: return launch_t<kEpiSwiglu>(a, num_sms, st);
        case kEpiBf16: return launch_t<kEpiBf16>(a, num_sms, st);
        case kEpiF32: return launch_t<kEpiF32>(a, num_sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace obs
