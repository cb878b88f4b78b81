// Fused attention on the tensor cores (tcgen05, 3xTF32): O = softmax(f(Q K^T)) V for
// one head per blockIdx.z and 128 query rows per CTA, online softmax over 64-key
// blocks. Needs the helpers of mt_tc.cuh. Head dim D = 64.
//
// Both products run as error-compensated TF32 (hi*hi + hi*lo + lo*hi, see mt_tc.cuh):
//   S_i = Q K_i^T   A = Q hi / lo in tensor memory (split once per CTA),
//                   B = K block (64 keys x 64 d, d contiguous: K-major), hi / lo in smem.
//   O_i = P_i V_i   A = P hi / lo in tensor memory (written by the softmax threads),
//                   B = V block (64 keys x 64 d, d contiguous: MN-major), hi / lo in smem.
// Every block's P V product lands in a fresh TMEM buffer and is added to the fp32
// output rows in registers (O = O * alpha + P_i V_i), so the tensor core's own fp32
// accumulation never runs longer than one 64-key block.
//
// Pipelining: S and the P V products are double buffered, P single buffered. The
// softmax of block i computes its exponentials while P V of block i - 1 and Q K of
// block i + 1 run; it waits for P V of block i - 1 only to overwrite P, writes P_i,
// and then folds P V of block i - 1 into the output (off the P -> P V critical path,
// while P V of block i and Q K of block i + 2 run). Shared memory carries only the K / V
// tiles: Q and P, the A operands, live in tensor memory.
//
// 512 threads, 16 warps:
//   warp 0       TMA producer (Q once, then K_i / V_i into a 2-stage ring) and Q K
//                issuer, in one non-blocking loop
//   warp 1       TMEM owner + P V issuer
//   warps 2..7   converters: split K_i and V_i into hi / lo in place
//   warps 8..15  softmax + output: thread = (query row = TMEM lane, half h of the
//                block's 64 keys and of the 64 output features); warp 8+q and 12+q
//                share lane quarter q. Warps 8..11 first split Q (row = lane) into
//                TMEM. Per block: read its 32 scores, exchange the half-row max with its
//                partner thread (smem + mbarrier), exponentiate, write its P hi / lo to
//                tensor memory, fold the previous block's P V into its 32 output
//                registers.
//
// Tensor memory (512 columns): Q hi/lo [0,128), S buffers [128,192) [192,256),
// P hi/lo [256,384), P V buffers [384,448) [448,512).
//
// Every wait is bounded (mt_mbar_wait); on a timeout the status word is set, every
// role leaves its loop, in-flight copies and MMAs are drained and the kernel returns.
#pragma once

struct mt_fa_layout {
    static constexpr uint32_t kQ = 0;                        // Q (TMA target): 2 k-tiles x 16 KB
    static constexpr uint32_t kStage0 = 32768;               // per stage: K hi, K lo, V hi, V lo (16 KB each)
    static constexpr uint32_t kStageBytes = 4u * 16384u;
    static constexpr uint32_t kXch = kStage0 + 2u * kStageBytes;    // float x[2 parity][2 half][128]
    static constexpr uint32_t kBar = kXch + 2u * 2u * 128u * 4u;
    static constexpr uint32_t kNumBars = 32;
    static constexpr uint32_t kBytes = kBar + kNumBars * 8u + 16u;
};

template <class ScoreFn>
__device__ __forceinline__ void mt_attn_fwd_tc(const mt_tmap* tmQ, const mt_tmap* tmK, const mt_tmap* tmV,
                                               float* __restrict__ O, float* __restrict__ row_max_out,
                                               float* __restrict__ row_sum_out, int Sq, int Sk, long long o_rs,
                                               const ScoreFn& f, int* status, void* smem_raw) {
    using L = mt_fa_layout;
    constexpr uint32_t QC = 0, SC = 128, PC = 256, OC = 384;
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* qfull = bars + 0;
    uint64_t* qconv = bars + 1;
    uint64_t* kfull = bars + 2;    // [2]
    uint64_t* vfull = bars + 4;    // [2]
    uint64_t* kconv = bars + 6;    // [2]
    uint64_t* vconv = bars + 8;    // [2]
    uint64_t* kempty = bars + 10;  // [2]
    uint64_t* vempty = bars + 12;  // [2]
    uint64_t* sfull = bars + 14;   // [2]
    uint64_t* sempty = bars + 16;  // [2]
    uint64_t* pfull = bars + 18;
    uint64_t* pempty = bars + 19;  // P V of the block done: P free, its product readable
    uint64_t* xbar = bars + 20;    // [4 quarters][2 parity]: half-row exchange
    uint64_t* mdone = bars + 28;   // P V issuer's MMAs drained
    uint64_t* pvi = bars + 29;     // [2] P V of the block issued (not done): Q K of block + 2 may follow
    uint64_t* qkdone = bars + 31;  // Q K issuer's MMAs drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xch = reinterpret_cast<float*>(smem + L::kXch);

    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    const int q0 = (int)blockIdx.x * 128, bz = (int)blockIdx.z;
    const int nb = Sk / 64;
    auto Qs = [&](int j) { return reinterpret_cast<float*>(smem + L::kQ + j * 16384); };
    auto Khi = [&](int s) { return reinterpret_cast<float*>(smem + L::kStage0 + s * L::kStageBytes); };
    auto Klo = [&](int s) { return reinterpret_cast<float*>(smem + L::kStage0 + s * L::kStageBytes + 16384); };
    auto Vhi = [&](int s) { return reinterpret_cast<float*>(smem + L::kStage0 + s * L::kStageBytes + 32768); };
    auto Vlo = [&](int s) { return reinterpret_cast<float*>(smem + L::kStage0 + s * L::kStageBytes + 49152); };

    if (threadIdx.x == 0) {
        // arrival counts: 1 = TMA expect_tx / tcgen05.commit, 4 = one lane per Q
        // splitting warp, 6 = one lane per converter warp, 8 = one lane per softmax
        // warp, 64 = every thread of a softmax warp pair
        for (int i = 0; i < 32; ++i) {
            const uint32_t n = i == 1 ? 4u : (i >= 6 && i <= 9) ? 6u : (i >= 16 && i <= 18) ? 8u
                             : (i >= 20 && i <= 27) ? 64u : 1u;
            mt_mbar_init(&bars[i], n);
        }
        *abort_flag = 0;
        mt_fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        mt_tma_prefetch(tmQ);
        mt_tma_prefetch(tmK);
        mt_tma_prefetch(tmV);
    }
    if (warp == 1) mt_tmem_alloc(tmem_slot, 512);
    mt_tc_fence_before();
    __syncthreads();
    mt_tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    constexpr uint32_t idesc_s = mt_idesc_tf32(128, 64, false, false);
    constexpr uint32_t idesc_o = mt_idesc_tf32(128, 64, false, true);
    if (warp == 0) {
        // TMA loads and the Q K products, in one non-blocking loop: each pass issues
        // whatever is ready (K_i once Q K of block i - 2 is done, V_i once P V of block
        // i - 2 is done, Q K of block j once K_j is split, S buffer j - 2 is read and
        // P V of block j - 2 is issued, which keeps P V ahead of the next Q K in the
        // tensor pipe). Issuing Q K here and P V from warp 1 lets one thread's barrier
        // waits overlap the other's MMAs (the tensor pipe queues almost nothing beyond
        // the MMA in flight, so a lone issuer idles it while it waits).
        if (lane == 0) {
            mt_mbar_expect_tx(qfull, 32768);
            mt_tma_load_3d(Qs(0), tmQ, qfull, 0, q0, bz);
            mt_tma_load_3d(Qs(1), tmQ, qfull, 32, q0, bz);
            int kl = 0, vl = 0, qk = 0;
            bool qready = false, issued_mma = false;
            uint64_t last = mt_globaltimer();
            for (uint32_t it = 1; kl < nb || vl < nb || qk < nb; ++it) {
                bool prog = false;
                if (kl < nb && (kl < 2 || mt_mbar_test(&kempty[kl & 1], (uint32_t)((kl >> 1) - 1) & 1u))) {
                    const int s = kl & 1;
                    mt_mbar_expect_tx(&kfull[s], 16384);
                    mt_tma_load_3d(Khi(s), tmK, &kfull[s], 0, kl * 64, bz);
                    mt_tma_load_3d(Khi(s) + 2048, tmK, &kfull[s], 32, kl * 64, bz);
                    ++kl;
                    prog = true;
                }
                if (vl < nb && (vl < 2 || mt_mbar_test(&vempty[vl & 1], (uint32_t)((vl >> 1) - 1) & 1u))) {
                    const int s = vl & 1;
                    mt_mbar_expect_tx(&vfull[s], 16384);
                    mt_tma_load_4d(Vhi(s), tmV, &vfull[s], 0, vl * 64, 0, bz);
                    mt_tma_load_4d(Vhi(s) + 2048, tmV, &vfull[s], 0, vl * 64 + 32, 0, bz);
                    ++vl;
                    prog = true;
                }
                if (qk < nb) {
                    const int s = qk & 1;
                    if (!qready) qready = mt_mbar_test(qconv, 0);
                    const uint32_t pprev = (uint32_t)((qk >> 1) - 1) & 1u;
                    if (qready && mt_mbar_test(&kconv[s], (uint32_t)(qk >> 1) & 1u) &&
                        (qk < 2 || (mt_mbar_test(&sempty[s], pprev) && mt_mbar_test(&pvi[s], pprev)))) {
                        mt_tc_fence_after();
                        const uint32_t d = tmem + SC + 64u * (uint32_t)s;
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            const uint32_t kh = mt_smem_u32(Khi(s) + j * 2048), kl2 = mt_smem_u32(Klo(s) + j * 2048);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint32_t ah = tmem + QC + 64u * (uint32_t)j + 8u * (uint32_t)kk;
                                const uint64_t bh = mt_operand_desc_k(kh, kk), bl = mt_operand_desc_k(kl2, kk);
                                mt_mma_tf32_ts(d, ah, bl, idesc_s, (j | kk) ? 1u : 0u);
                                mt_mma_tf32_ts(d, ah + 32u, bh, idesc_s, 1u);
                                mt_mma_tf32_ts(d, ah, bh, idesc_s, 1u);
                            }
                        }
                        mt_mma_commit(&kempty[s]);
                        mt_mma_commit(&sfull[s]);
                        issued_mma = true;
                        ++qk;
                        prog = true;
                    }
                }
                if (prog) {
                    last = mt_globaltimer();
                    continue;
                }
                __nanosleep(20);  // leave issue slots to the softmax warps sharing this scheduler
                if ((it & 63u) == 0) {
                    if (*abort_flag) break;
                    if (mt_globaltimer() - last > MT_WAIT_LIMIT_NS) {
                        atomicCAS(status, 0, 1);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            if (issued_mma) {  // all Q K products complete before TMEM can be released (bounded)
                mt_mma_commit(qkdone);
                mt_mbar_drain(qkdone, 0);
            }
            if (*abort_flag) {  // let this CTA's own copies land before it can exit
                mt_mbar_drain(qfull, 0);
                for (int i = (kl > 2 ? kl - 2 : 0); i < kl; ++i) mt_mbar_drain(&kfull[i & 1], (uint32_t)(i >> 1) & 1u);
                for (int i = (vl > 2 ? vl - 2 : 0); i < vl; ++i) mt_mbar_drain(&vfull[i & 1], (uint32_t)(i >> 1) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < nb && ok; ++i) {
                const int s = i & 1;
                // pfull(i) also means the softmax threads have folded P V of block i - 2
                // out of this block's P V buffer
                if (!mt_mbar_wait(pfull, (uint32_t)i & 1u, abort_flag, status, 2)) break;
                if (!mt_mbar_wait(&vconv[s], (uint32_t)(i >> 1) & 1u, abort_flag, status, 2)) break;
                mt_tc_fence_after();
                const uint32_t d = tmem + OC + 64u * (uint32_t)s;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint32_t vh = mt_smem_u32(Vhi(s) + j * 2048), vl = mt_smem_u32(Vlo(s) + j * 2048);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t ah = tmem + PC + 64u * (uint32_t)j + 8u * (uint32_t)kk;
                        const uint64_t bh = mt_operand_desc_mn(vh, kk), bl = mt_operand_desc_mn(vl, kk);
                        mt_mma_tf32_ts(d, ah, bl, idesc_o, (j | kk) ? 1u : 0u);
                        mt_mma_tf32_ts(d, ah + 32u, bh, idesc_o, 1u);
                        mt_mma_tf32_ts(d, ah, bh, idesc_o, 1u);
                    }
                }
                mt_mma_commit(&vempty[s]);
                mt_mma_commit(pempty);
                mt_mbar_arrive(&pvi[s]);
            }
            // All issued MMAs complete before TMEM can be released (bounded).
            mt_mma_commit(mdone);
            mt_mbar_drain(mdone, 0);
        }
    } else if (warp < 8) {
        const int ct = (warp - 2) * 32 + lane;
        const mt_no_prologue np{};
        for (int i = 0; i < nb; ++i) {
            const int s = i & 1;
            const uint32_t par = (uint32_t)(i >> 1) & 1u;
            if (!mt_mbar_wait(&kfull[s], par, abort_flag, status, 3)) break;
            mt_convert_tile<false, false, 128, 192>(Khi(s), Khi(s), Klo(s), 0, 0, 0, 0, np, ct);
            mt_fence_proxy_async();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive(&kconv[s]);
            if (!mt_mbar_wait(&vfull[s], par, abort_flag, status, 3)) break;
            mt_convert_tile<false, false, 128, 192>(Vhi(s), Vhi(s), Vlo(s), 0, 0, 0, 0, np, ct);
            mt_fence_proxy_async();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive(&vconv[s]);
        }
    } else {
        const int q = warp & 3, h = (warp - 8) >> 2, r = q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        bool ok = true;
        if (h == 0) {
            ok = mt_mbar_wait(qfull, 0, abort_flag, status, 4);
            if (ok) {
                const mt_no_prologue np{};
                mt_convert_a_rows(Qs(0), tmem + QC, q, lane, 0, 0, 0, 0, np);
                mt_convert_a_rows(Qs(1), tmem + QC + 64u, q, lane, 0, 0, 0, 0, np);
                mt_tc_fence_before();
                __syncwarp();
                if (lane == 0) mt_mbar_arrive(qconv);
            }
        }
        // half-row exchange with the partner thread (same row, other half)
        auto exchange = [&](int blk, float v) -> float {
            const int par = blk & 1;
            xch[(par * 2 + h) * 128 + r] = v;
            mt_mbar_arrive(&xbar[q * 2 + par]);
            if (!mt_mbar_wait(&xbar[q * 2 + par], (uint32_t)(blk >> 1) & 1u, abort_flag, status, 4)) {
                ok = false;
                return v;
            }
            return xch[(par * 2 + (h ^ 1)) * 128 + r];
        };
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.0f;
        // fold P V of block `blk` (finished: its pempty waited) into the output registers
        auto fold = [&](int blk, float alpha) {
            mt_tc_fence_after();
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float t[16];
                mt_tmem_ld16(tmem + lane_off + OC + 64u * (uint32_t)(blk & 1) + 32u * (uint32_t)h +
                                 16u * (uint32_t)hh, t);
#pragma unroll
                for (int j = 0; j < 16; ++j) o[16 * hh + j] = fmaf(o[16 * hh + j], alpha, t[j]);
            }
        };
        float m = -INFINITY, l = 0.0f;
        float a_prev = 0.0f;  // alpha of the previous block
        for (int i = 0; i < nb && ok; ++i) {
            const int s = i & 1;
            if (!mt_mbar_wait(&sfull[s], (uint32_t)(i >> 1) & 1u, abort_flag, status, 4)) {
                ok = false;
                break;
            }
            mt_tc_fence_after();
            float sv[32];
            mt_tmem_ld32(tmem + lane_off + SC + 64u * (uint32_t)s + 32u * (uint32_t)h, sv);
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive(&sempty[s]);
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                sv[j] = f(sv[j]);
                mx[j & 3] = fmaxf(mx[j & 3], sv[j]);
            }
            float bm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            bm = fmaxf(bm, exchange(i, bm));
            if (!ok) break;
            const float mn = fmaxf(m, bm);
            const float alpha = (m == -INFINITY) ? 0.0f : expf(__fsub_rn(m, mn));
            float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                // exp of a non-positive argument: the MUFU ex2-based intrinsic; the
                // normwise error of O is unchanged against expf (9.8e-7 vs 9.8e-7 at
                // 4 x 512 x 64) and the block runs ~10% faster
                const float p = (sv[j] == -INFINITY) ? 0.0f : __expf(__fsub_rn(sv[j], mn));
                sv[j] = p;
                ps[j & 3] = __fadd_rn(ps[j & 3], p);
            }
            l = fmaf(l, alpha, __fadd_rn(__fadd_rn(ps[0], ps[1]), __fadd_rn(ps[2], ps[3])));
            m = mn;
            // P V of block i - 1 done: P is free (its product is folded below)
            if (i >= 1 && !mt_mbar_wait(pempty, (uint32_t)(i - 1) & 1u, abort_flag, status, 4)) {
                ok = false;
                break;
            }
            mt_tc_fence_after();
            const uint32_t pbuf = tmem + lane_off + PC + 64u * (uint32_t)h;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float lo[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float x = sv[16 * hh + k];
                    mt_split_tf32(x, sv[16 * hh + k], lo[k]);
                }
                mt_tmem_st16_nowait(pbuf + 16u * (uint32_t)hh, &sv[16 * hh]);
                mt_tmem_st16_nowait(pbuf + 32u + 16u * (uint32_t)hh, lo);
                mt_tmem_wait_st();  // before `lo` is refilled
            }
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive(pfull);
            // P V of block i - 1 into the output, while P V of block i runs; its TMEM
            // buffer is next written by P V of block i + 1, after pfull(i + 1)
            if (i >= 1) fold(i - 1, a_prev);
            a_prev = alpha;
        }
        if (ok && mt_mbar_wait(pempty, (uint32_t)(nb - 1) & 1u, abort_flag, status, 4)) fold(nb - 1, a_prev);
        else ok = false;
        if (ok) {
            const float lt = __fadd_rn(l, exchange(nb, l));
            const int row = q0 + r;
            if (ok && row < Sq) {
                const float inv = __fdiv_rn(1.0f, lt);
                float4* dst = reinterpret_cast<float4*>(O + (long long)row * o_rs + 32 * h);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    dst[j] = make_float4(o[4 * j] * inv, o[4 * j + 1] * inv, o[4 * j + 2] * inv, o[4 * j + 3] * inv);
                if (h == 0) {
                    if (row_max_out) row_max_out[row] = m;
                    if (row_sum_out) row_sum_out[row] = lt;
                }
            }
        }
    }
    mt_tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        mt_tc_fence_after();
        mt_tmem_dealloc(tmem, 512);
    }
}
