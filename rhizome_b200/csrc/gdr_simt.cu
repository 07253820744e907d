// SIMT kernels of the GDR library (sm_100a):
//   - gdr_step_kernel: one position of the recurrence for a ragged batch of
//     sequences whose states live in a slot pool (decode, memory bound);
//   - gdr_seq_kernel: the recurrence applied position by position over whole
//     sequences in fp32 (the rtol-1e-5 path, and the path for head widths the
//     tensor-core kernel does not tile).
//
// Both follow gated_delta_step (crates/ops/src/delta.rs:93-127) per row:
//   sk_i = sum_j S_ij k_j
//   S_ij <- alpha (S_ij - (beta sk_i) k_j) + (beta v_i) k_j
//   o_i  = sum_j S_ij q_j
// Rows (the v index i) are independent, so a (sequence, head) can be split
// into row blocks across warps and CTAs with no cross-CTA reduction.
//
// Register layout: a warp owns RPW consecutive rows; lane l owns the column
// vectors j = 128 c + 4 l + e (c < NV, e < 4). A row's partial dot products
// are combined with a transposing butterfly: RPW values per lane are halved
// at each of the first log2(RPW) xor-shuffle levels, so the sums of 16 rows
// cost 16 shuffles (plus 16 to broadcast them back) instead of 5 per row.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace rhz {
namespace {

constexpr unsigned FULL = 0xffffffffu;

template <int N> struct Log2 { static constexpr int value = 1 + Log2<N / 2>::value; };
template <> struct Log2<1> { static constexpr int value = 0; };

// After the call, v[0] on lane l holds the full 32-lane sum of row
// (l >> (5 - log2 N)); every lane of that row's group holds it.
template <int N>
__device__ __forceinline__ void transpose_reduce(float (&v)[N], int lane) {
#pragma unroll
    for (int half = N / 2, off = 16; half >= 1; half /= 2, off /= 2) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            float send = upper ? v[i] : v[i + half];
            float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(FULL, send, off);
        }
    }
#pragma unroll
    for (int off = 16 >> Log2<N>::value; off >= 1; off /= 2) v[0] += __shfl_xor_sync(FULL, v[0], off);
}

// Row sums of s[r][.] . x[.] for this warp's RPW rows. Returns (via out[r])
// the full sum of every row on every lane; `mine` gets the sum of the row
// this lane represents (row index lane >> SHIFT).
template <int RPW, int NV>
__device__ __forceinline__ void row_dots(const float (&s)[RPW][NV][4], const float (&x)[NV][4],
                                         int lane, float (&out)[RPW], float &mine) {
    float p[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < NV; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = fmaf(s[r][c][e], x[c][e], acc);
        p[r] = acc;
    }
    transpose_reduce<RPW>(p, lane);
    mine = p[0];
    constexpr int SHIFT = 5 - Log2<RPW>::value;
#pragma unroll
    for (int r = 0; r < RPW; ++r) out[r] = __shfl_sync(FULL, p[0], r << SHIFT);
}

template <int RPW, int NV>
__device__ __forceinline__ void rank1_update(float (&s)[RPW][NV][4], const float (&kk)[NV][4],
                                             const float (&sk)[RPW], const float (&vr)[RPW],
                                             float a, float b) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const float bsk = b * sk[r];
        const float bv = b * vr[r];
#pragma unroll
        for (int c = 0; c < NV; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float decayed = a * (s[r][c][e] - bsk * kk[c][e]);
                s[r][c][e] = decayed + bv * kk[c][e];
            }
    }
}

__device__ __forceinline__ int nvalid(int d, int j) {
    int n = d - j;
    return n < 0 ? 0 : (n > 4 ? 4 : n);
}

// ------------------------------------------------------------------ decode

template <typename T, int RPW, int NV, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    gdr_step_kernel(T *__restrict__ o, float *__restrict__ pool, const int32_t *__restrict__ slots,
                    const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
                    const float *__restrict__ alpha, const float *__restrict__ beta,
                    int64_t num_slots, int H, int d, bool vec) {
    const int64_t item = blockIdx.x;  // sequence * H + head
    const int64_t seq = item / H;
    const int h = static_cast<int>(item - seq * H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.y * (WARPS * RPW) + warp * RPW;
    if (row0 >= d) return;
    constexpr int SHIFT = 5 - Log2<RPW>::value;
    const int myrow = row0 + (lane >> SHIFT);
    const bool writer = (lane & ((1 << SHIFT) - 1)) == 0 && myrow < d;

    const int64_t slot = slots ? static_cast<int64_t>(slots[seq]) : seq;
    T *op = o + item * d;
    if (slot < 0 || slot >= num_slots) {
        if (writer) op[myrow] = from_f32<T>(nanf(""));
        return;
    }
    const T *qp = q + item * d, *kp = k + item * d, *vp = v + item * d;
    float *S = pool + (static_cast<int64_t>(slot) * H + h) * static_cast<int64_t>(d) * d;

    float s[RPW][NV][4];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int row = row0 + r;
#pragma unroll
        for (int c = 0; c < NV; ++c) {
            const int j = 128 * c + 4 * lane;
            if (row < d) {
                load4(S + static_cast<int64_t>(row) * d + j, vec, nvalid(d, j), s[r][c]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) s[r][c][e] = 0.f;
            }
        }
    }
    float kk[NV][4], qq[NV][4], vr[RPW];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = 128 * c + 4 * lane;
        load4(kp + j, vec, nvalid(d, j), kk[c]);
        load4(qp + j, vec, nvalid(d, j), qq[c]);
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) vr[r] = row0 + r < d ? to_f32(vp[row0 + r]) : 0.f;
    const float a = alpha[item], b = beta[item];

    float sk[RPW], mine;
    row_dots<RPW, NV>(s, kk, lane, sk, mine);
    rank1_update<RPW, NV>(s, kk, sk, vr, a, b);
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int row = row0 + r;
        if (row < d) {
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                const int j = 128 * c + 4 * lane;
                store4(S + static_cast<int64_t>(row) * d + j, vec, nvalid(d, j), s[r][c]);
            }
        }
    }
    float ov[RPW];
    row_dots<RPW, NV>(s, qq, lane, ov, mine);
    if (writer) op[myrow] = from_f32<T>(mine);
}

// ------------------------------------------------------------------ multistep

// gated_delta_multistep (delta.rs:201-230) for n sequences x H heads of up
// to Tn positions: the state rows stay in registers across the positions and
// the state after every position is written out (speculative decoding keeps
// them to roll back to the last accepted draft token). With pool == nullptr
// the state starts at zero and resets wherever the segment id changes (the
// reference's semantics; its reset at t = 0 discards `init`); otherwise it
// starts from pool[slot] and the pool is left untouched.
template <typename T, int RPW, int NV, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    gdr_multistep_kernel(T *__restrict__ outs, float *__restrict__ states,
                         const float *__restrict__ pool, const int32_t *__restrict__ slots,
                         const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
                         const float *__restrict__ alpha, const float *__restrict__ beta,
                         const int64_t *__restrict__ segment, int64_t Tin, int Tn,
                         int64_t num_slots, int H, int d, bool vec) {
    const int64_t item = blockIdx.x;  // sequence * H + head
    const int64_t seq = item / H;
    const int h = static_cast<int>(item - seq * H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.y * (WARPS * RPW) + warp * RPW;
    if (row0 >= d) return;
    constexpr int SHIFT = 5 - Log2<RPW>::value;
    const int myrow = row0 + (lane >> SHIFT);
    const bool writer = (lane & ((1 << SHIFT) - 1)) == 0 && myrow < d;
    const int64_t dd = static_cast<int64_t>(d) * d;

    float s[RPW][NV][4];
    bool valid = true;
    if (pool) {
        const int64_t slot = slots ? static_cast<int64_t>(slots[seq]) : seq;
        valid = slot >= 0 && slot < num_slots;
        const float *S = valid ? pool + (slot * H + h) * dd : nullptr;
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                const int j = 128 * c + 4 * lane;
                if (valid && row0 + r < d) {
                    load4(S + static_cast<int64_t>(row0 + r) * d + j, vec, nvalid(d, j), s[r][c]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[r][c][e] = 0.f;
                }
            }
    } else {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int c = 0; c < NV; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[r][c][e] = 0.f;
    }
    const int64_t row_stride = static_cast<int64_t>(H) * d;
    for (int t = 0; t < Tn; ++t) {
        const int64_t tok = seq * Tin + t;
        if (!pool && segment && t > 0 && segment[tok] != segment[tok - 1]) {
#pragma unroll
            for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int c = 0; c < NV; ++c)
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[r][c][e] = 0.f;
        }
        const T *qp = q + tok * row_stride + static_cast<int64_t>(h) * d;
        const T *kp = k + tok * row_stride + static_cast<int64_t>(h) * d;
        const T *vp = v + tok * row_stride + static_cast<int64_t>(h) * d;
        float kk[NV][4], qq[NV][4], vr[RPW];
#pragma unroll
        for (int c = 0; c < NV; ++c) {
            const int j = 128 * c + 4 * lane;
            load4(kp + j, vec, nvalid(d, j), kk[c]);
            load4(qp + j, vec, nvalid(d, j), qq[c]);
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) vr[r] = row0 + r < d ? to_f32(vp[row0 + r]) : 0.f;
        const float a = alpha[tok * H + h], b = beta[tok * H + h];
        float sk[RPW], ov[RPW], mine;
        row_dots<RPW, NV>(s, kk, lane, sk, mine);
        rank1_update<RPW, NV>(s, kk, sk, vr, a, b);
        row_dots<RPW, NV>(s, qq, lane, ov, mine);
        T *op = outs + (seq * Tn + t) * row_stride + static_cast<int64_t>(h) * d;
        if (writer) op[myrow] = valid ? from_f32<T>(mine) : from_f32<T>(nanf(""));
        float *St = states + ((seq * Tn + t) * H + h) * dd;
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            if (row0 + r < d) {
#pragma unroll
                for (int c = 0; c < NV; ++c) {
                    const int j = 128 * c + 4 * lane;
                    store4(St + static_cast<int64_t>(row0 + r) * d + j, vec, nvalid(d, j), s[r][c]);
                }
            }
        }
    }
}

// ------------------------------------------------------------------ sequential

// Tile of TS positions staged in shared memory: k and q rows (all d
// columns), the CTA's v rows, alpha and beta.
template <typename T, int ROWS, int TS>
struct SeqTile {
    static size_t bytes(int d) {
        return (size_t(2) * TS * d + size_t(TS) * ROWS) * sizeof(float) + 2 * TS * sizeof(float);
    }
};

template <typename T, int RPW, int NV, int WARPS, int TS>
__global__ void __launch_bounds__(WARPS * 32)
    gdr_seq_kernel(T *__restrict__ o, const T *__restrict__ q, const T *__restrict__ k,
                   const T *__restrict__ v, const float *__restrict__ alpha,
                   const float *__restrict__ beta, const int32_t *__restrict__ cu_seqlens,
                   const int32_t *__restrict__ n_seq_dev, int64_t n_seq_host, int64_t seq_len,
                   int64_t total_tokens,
                   const float *__restrict__ state_in, const int32_t *__restrict__ in_slots,
                   float *__restrict__ state_out, const int32_t *__restrict__ out_slots,
                   int64_t num_slots, int H, int d, bool vec) {
    constexpr int ROWS = WARPS * RPW;
    constexpr int SHIFT = 5 - Log2<RPW>::value;
    extern __shared__ float4 smem_raw[];
    float *smem = reinterpret_cast<float *>(smem_raw);
    float *sk_ = smem;                       // [TS][d]
    float *sq_ = sk_ + TS * d;               // [TS][d]
    float *sv_ = sq_ + TS * d;               // [TS][ROWS]
    float *sa_ = sv_ + TS * ROWS;            // [TS]
    float *sb_ = sa_ + TS;                   // [TS]
    const int nthr = WARPS * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rb0 = blockIdx.y * ROWS;
    const int row0 = rb0 + warp * RPW;
    const int myrow = row0 + (lane >> SHIFT);
    const bool writer = (lane & ((1 << SHIFT) - 1)) == 0 && myrow < d;
    const int64_t row_stride = static_cast<int64_t>(H) * d;  // token stride in q/k/v/o

    int64_t n_seq = n_seq_host;
    if (n_seq_dev) {
        const int64_t nd = *n_seq_dev;
        n_seq = nd < n_seq ? nd : n_seq;
    }
    const int64_t n_items = n_seq * H;

    // Persistent loop over (sequence, head) items; all threads of the CTA
    // take the same item, so the barriers below stay uniform.
    for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int64_t seq = item / H;
        const int h = static_cast<int>(item - seq * H);
        int64_t t0, t1;
        if (cu_seqlens) {
            // Offsets are caller data: clamp them to the packed stream.
            t0 = cu_seqlens[seq];
            t1 = cu_seqlens[seq + 1];
            t0 = t0 < 0 ? 0 : (t0 > total_tokens ? total_tokens : t0);
            t1 = t1 < t0 ? t0 : (t1 > total_tokens ? total_tokens : t1);
        } else {
            t0 = seq * seq_len;
            t1 = t0 + seq_len;
        }

        // Initial state rows: zeros unless state_in is given (the reset at a
        // segment start, delta.rs:139-141, is the zero case).
        float s[RPW][NV][4];
        int64_t in_slot = -1;
        if (state_in) in_slot = in_slots ? static_cast<int64_t>(in_slots[seq]) : seq;
        const bool have_in = state_in && in_slot >= 0 && in_slot < num_slots;
        const float *Sin =
            have_in ? state_in + (in_slot * H + h) * static_cast<int64_t>(d) * d : nullptr;
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int row = row0 + r;
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                const int j = 128 * c + 4 * lane;
                if (have_in && row < d) {
                    load4(Sin + static_cast<int64_t>(row) * d + j, vec, nvalid(d, j), s[r][c]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[r][c][e] = 0.f;
                }
            }
        }

        for (int64_t tt = t0; tt < t1; tt += TS) {
            const int n = static_cast<int>((t1 - tt) < TS ? (t1 - tt) : TS);
            __syncthreads();
            for (int idx = threadIdx.x; idx < n * d; idx += nthr) {
                const int t = idx / d, j = idx - t * d;
                const int64_t g = (tt + t) * row_stride + static_cast<int64_t>(h) * d + j;
                sk_[t * d + j] = to_f32(k[g]);
                sq_[t * d + j] = to_f32(q[g]);
            }
            for (int idx = threadIdx.x; idx < n * ROWS; idx += nthr) {
                const int t = idx / ROWS, r = idx - t * ROWS;
                const int row = rb0 + r;
                sv_[t * ROWS + r] =
                    row < d ? to_f32(v[(tt + t) * row_stride + static_cast<int64_t>(h) * d + row])
                            : 0.f;
            }
            for (int t = threadIdx.x; t < n; t += nthr) {
                sa_[t] = alpha[(tt + t) * H + h];
                sb_[t] = beta[(tt + t) * H + h];
            }
            __syncthreads();
            if (row0 < d) {
                for (int t = 0; t < n; ++t) {
                    float kk[NV][4], qq[NV][4], vr[RPW];
#pragma unroll
                    for (int c = 0; c < NV; ++c) {
                        const int j = 128 * c + 4 * lane;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const bool ok = j + e < d;
                            kk[c][e] = ok ? sk_[t * d + j + e] : 0.f;
                            qq[c][e] = ok ? sq_[t * d + j + e] : 0.f;
                        }
                    }
#pragma unroll
                    for (int r = 0; r < RPW; ++r) vr[r] = sv_[t * ROWS + warp * RPW + r];
                    float sk[RPW], ov[RPW], mine;
                    row_dots<RPW, NV>(s, kk, lane, sk, mine);
                    rank1_update<RPW, NV>(s, kk, sk, vr, sa_[t], sb_[t]);
                    row_dots<RPW, NV>(s, qq, lane, ov, mine);
                    if (writer) {
                        o[(tt + t) * row_stride + static_cast<int64_t>(h) * d + myrow] =
                            from_f32<T>(mine);
                    }
                }
            }
        }

        if (state_out && row0 < d) {
            const int64_t out_slot = out_slots ? static_cast<int64_t>(out_slots[seq]) : seq;
            if (out_slot >= 0 && out_slot < num_slots) {
                float *Sout = state_out + (out_slot * H + h) * static_cast<int64_t>(d) * d;
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    const int row = row0 + r;
                    if (row < d) {
#pragma unroll
                        for (int c = 0; c < NV; ++c) {
                            const int j = 128 * c + 4 * lane;
                            store4(Sout + static_cast<int64_t>(row) * d + j, vec, nvalid(d, j),
                                   s[r][c]);
                        }
                    }
                }
            }
        }
    }
}

template <typename T, int RPW, int NV, int WARPS>
int launch_step_t(const StepArgs &a) {
    dim3 grid(static_cast<unsigned>(a.n * a.H), (a.d + WARPS * RPW - 1) / (WARPS * RPW));
    const bool vec = (a.d % 4) == 0;
    gdr_step_kernel<T, RPW, NV, WARPS><<<grid, WARPS * 32, 0, a.stream>>>(
        static_cast<T *>(a.o), a.pool, a.slots, static_cast<const T *>(a.q),
        static_cast<const T *>(a.k), static_cast<const T *>(a.v), a.alpha, a.beta, a.num_slots,
        a.H, a.d, vec);
    return check_launch("gdr_step_kernel");
}

template <typename T, int RPW, int NV, int WARPS, int TS>
int launch_seq_t(const SeqArgs &a) {
    constexpr int ROWS = WARPS * RPW;
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    const int64_t items = a.n_seq * a.H;
    const int row_blocks = (a.d + ROWS - 1) / ROWS;
    // Enough CTAs to fill every SM a few times over; the kernel loops over the
    // remaining (sequence, head) items.
    int64_t gx = static_cast<int64_t>(sms) * 16 / row_blocks;
    if (gx < 1) gx = 1;
    if (gx > items) gx = items;
    dim3 grid(static_cast<unsigned>(gx), row_blocks);
    const size_t smem = SeqTile<T, ROWS, TS>::bytes(a.d);
    auto kern = gdr_seq_kernel<T, RPW, NV, WARPS, TS>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "gdr_seq_kernel smem: %s", cudaGetErrorString(e));
    }
    const bool vec = (a.d % 4) == 0;
    kern<<<grid, WARPS * 32, smem, a.stream>>>(
        static_cast<T *>(a.o), static_cast<const T *>(a.q), static_cast<const T *>(a.k),
        static_cast<const T *>(a.v), a.alpha, a.beta, a.cu_seqlens, a.n_seq_dev, a.n_seq, a.seq_len,
        a.cu_seqlens ? a.total_tokens : a.n_seq * a.seq_len,
        a.state_in, a.in_slots, a.state_out, a.out_slots, a.num_slots, a.H, a.d, vec);
    return check_launch("gdr_seq_kernel");
}

template <typename T, int RPW, int NV, int WARPS>
int launch_multistep_t(const MultistepArgs &a) {
    dim3 grid(static_cast<unsigned>(a.n * a.H), (a.d + WARPS * RPW - 1) / (WARPS * RPW));
    const bool vec = (a.d % 4) == 0;
    gdr_multistep_kernel<T, RPW, NV, WARPS><<<grid, WARPS * 32, 0, a.stream>>>(
        static_cast<T *>(a.outs), a.states, a.pool, a.slots, static_cast<const T *>(a.q),
        static_cast<const T *>(a.k), static_cast<const T *>(a.v), a.alpha, a.beta, a.segment,
        a.T, a.Tn, a.num_slots, a.H, a.d, vec);
    return check_launch("gdr_multistep_kernel");
}

}  // namespace

int launch_multistep(const MultistepArgs &a) {
    if (a.n == 0 || a.Tn == 0) return RHZ_OK;
    if (a.dtype == RHZ_DTYPE_BF16) {
        if (a.d <= 128) return launch_multistep_t<__nv_bfloat16, 8, 1, 8>(a);
        return launch_multistep_t<__nv_bfloat16, 4, 2, 8>(a);
    }
    if (a.d <= 128) return launch_multistep_t<float, 8, 1, 8>(a);
    return launch_multistep_t<float, 4, 2, 8>(a);
}

int launch_step(const StepArgs &a) {
    if (a.n == 0) return RHZ_OK;
    // d <= 128: one vector column per lane; 129..256: two. 64 rows per CTA
    // keep registers near 64/thread so three CTAs (96 KB of state loads in
    // flight) share an SM.
    if (a.dtype == RHZ_DTYPE_BF16) {
        if (a.d <= 128) return launch_step_t<__nv_bfloat16, 8, 1, 8>(a);
        return launch_step_t<__nv_bfloat16, 4, 2, 8>(a);
    }
    if (a.d <= 128) return launch_step_t<float, 8, 1, 8>(a);
    return launch_step_t<float, 4, 2, 8>(a);
}

int launch_seq(const SeqArgs &a) {
    if (a.n_seq == 0) return RHZ_OK;
    if (a.dtype == RHZ_DTYPE_BF16) {
        if (a.d <= 128) return launch_seq_t<__nv_bfloat16, 4, 1, 4, 32>(a);
        return launch_seq_t<__nv_bfloat16, 4, 2, 4, 16>(a);
    }
    if (a.d <= 128) return launch_seq_t<float, 4, 1, 4, 32>(a);
    return launch_seq_t<float, 4, 2, 4, 16>(a);
}

}  // namespace rhz
