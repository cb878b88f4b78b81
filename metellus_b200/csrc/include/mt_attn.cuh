// Fused attention (FFMA pipe): O = softmax(f(Q K^T)) V for one head per blockIdx.z,
// 64 query rows per CTA, online softmax over 64-key blocks (the S x S score matrix is
// never materialised). `f` is the lane-agnostic score chain of the program (e.g. the
// 0.125 scale). Also writes the per-row statistics the program declares: the row max
// of f(QK^T) and the row sum of exp(f(QK^T) - max).
//
// 256 threads: thread (ty, tx) = (tid / 16, tid % 16) owns rows 4ty..4ty+3 and score
// columns / output features 4tx..4tx+3. Shared tiles are stored transposed where that
// makes the inner-product reads 128-bit and conflict free.
#pragma once

template <int D>
struct mt_attn_smem {
    static constexpr int BQ = 64, BK = 64, P = 4;
    static constexpr int kQ = D * (BQ + P);     // Qs[d][q]
    static constexpr int kK = D * (BK + P);     // Ks[d][key]
    static constexpr int kV = BK * (D + P);     // Vs[key][d]
    static constexpr int kP = BK * (BQ + P);    // Ps[key][q]
    static constexpr int kFloats = kQ + kK + kV + kP;
};

template <int D, class ScoreFn>
__device__ __forceinline__ void mt_attn_fwd_simt(const float* __restrict__ Q, const float* __restrict__ Kp,
                                                 const float* __restrict__ V, float* __restrict__ O,
                                                 float* __restrict__ row_max_out, float* __restrict__ row_sum_out,
                                                 int Sq, int Sk, long long q_rs, long long k_rs, long long v_rs,
                                                 long long o_rs, const ScoreFn& f, float* smem) {
    static_assert(D % 64 == 0 && D <= 128, "head dim must be 64 or 128");
    using L = mt_attn_smem<D>;
    constexpr int BQ = L::BQ, BK = L::BK, P = L::P;
    constexpr int DG = D / 64;  // groups of 64 output features; thread tx owns 4 per group
    float* Qs = smem;
    float* Ks = Qs + L::kQ;
    float* Vs = Ks + L::kK;
    float* Ps = Vs + L::kV;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int q0 = blockIdx.x * BQ;

    // Q tile, transposed: Qs[d][q]
    for (int i = tid; i < BQ * D; i += 256) {
        const int q = i / D, d = i % D;
        Qs[d * (BQ + P) + q] = (q0 + q < Sq) ? Q[(long long)(q0 + q) * q_rs + d] : 0.0f;
    }
    float m[4], l[4];
    float o[4][DG][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < DG; ++c)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][c][j] = 0.0f;
    }
    for (int k0 = 0; k0 < Sk; k0 += BK) {
        __syncthreads();
        for (int i = tid; i < BK * D; i += 256) {
            const int kk = i / D, d = i % D;
            const bool ok = k0 + kk < Sk;
            Ks[d * (BK + P) + kk] = ok ? Kp[(long long)(k0 + kk) * k_rs + d] : 0.0f;
            Vs[kk * (D + P) + d] = ok ? V[(long long)(k0 + kk) * v_rs + d] : 0.0f;
        }
        __syncthreads();
        float s[4][4] = {};
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
            const float4 a = *reinterpret_cast<const float4*>(&Qs[d * (BQ + P) + 4 * ty]);
            const float4 b = *reinterpret_cast<const float4*>(&Ks[d * (BK + P) + 4 * tx]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float bm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[i][j] = (k0 + 4 * tx + j < Sk) ? f(s[i][j]) : -INFINITY;
                bm = fmaxf(bm, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
            const float mn = fmaxf(m[i], bm);
            const float alpha = (m[i] == -INFINITY) ? 0.0f : expf(__fsub_rn(m[i], mn));
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = (s[i][j] == -INFINITY) ? 0.0f : expf(__fsub_rn(s[i][j], mn));
                s[i][j] = p;
                rs = __fadd_rn(rs, p);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs = __fadd_rn(rs, __shfl_xor_sync(0xffffffffu, rs, off));
            l[i] = fmaf(l[i], alpha, rs);
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < DG; ++c)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[i][c][j] *= alpha;
        }
        // P transposed: Ps[key][q]
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float4 col = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
            *reinterpret_cast<float4*>(&Ps[(4 * tx + j) * (BQ + P) + 4 * ty]) = col;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < BK; ++kk) {
            const float4 p = *reinterpret_cast<const float4*>(&Ps[kk * (BQ + P) + 4 * ty]);
            const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (int c = 0; c < DG; ++c) {
                const float4 v = *reinterpret_cast<const float4*>(&Vs[kk * (D + P) + 64 * c + 4 * tx]);
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) o[i][c][j] = fmaf(pv[i], vv[j], o[i][c][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = q0 + 4 * ty + i;
        if (q >= Sq) continue;
        const float inv = __fdiv_rn(1.0f, l[i]);
#pragma unroll
        for (int c = 0; c < DG; ++c) {
            float4 r = make_float4(o[i][c][0] * inv, o[i][c][1] * inv, o[i][c][2] * inv, o[i][c][3] * inv);
            *reinterpret_cast<float4*>(&O[(long long)q * o_rs + 64 * c + 4 * tx]) = r;
        }
        if (tx == 0) {
            if (row_max_out) row_max_out[q] = m[i];
            if (row_sum_out) row_sum_out[q] = l[i];
        }
    }
}
