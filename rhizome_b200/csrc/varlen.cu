// Variable-length packing kernels (index and byte work, bit-exact):
// cu_seqlens prefix sums, segment ids -> boundaries, chunk maps, slot-pool
// state gather/scatter and padded <-> packed token moves. They give
// continuous-batched prefill and decode one packed layout: sequence i owns
// token rows [cu_seqlens[i], cu_seqlens[i+1]) and state slot slot_idx[i].
//
// All of it is HBM or latency bound integer work. Scans are block-local
// (warp shuffles + one shared-memory pass) with a grid-wide three-phase
// scheme (tile totals -> one-CTA scan of the totals -> tile scan + offset)
// whose only scratch is one int32 per tile, passed in as workspace.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace rhz {
namespace {

constexpr int SCAN_THREADS = 512;
constexpr int SCAN_ITEMS = 8;                        // items per thread
constexpr int SCAN_TILE = SCAN_THREADS * SCAN_ITEMS; // 4096 items per tile

// Exclusive scan of one int per thread across the CTA; returns the CTA total
// through `total`. `warp_sums` needs SCAN_THREADS / 32 ints.
__device__ __forceinline__ int block_exclusive_scan(int x, int *warp_sums, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        constexpr int NW = SCAN_THREADS / 32;
        int w = lane < NW ? warp_sums[lane] : 0;
        int wi = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, wi, off);
            if (lane >= off) wi += y;
        }
        if (lane < NW) warp_sums[lane] = wi - w;  // exclusive warp offsets
        if (lane == NW - 1) warp_sums[NW] = wi;   // CTA total
    }
    __syncthreads();
    const int res = warp_sums[warp] + incl - x;
    total = warp_sums[SCAN_THREADS / 32];
    __syncthreads();
    return res;
}

// ---- segment ids -> boundaries

__device__ __forceinline__ int seg_flag(const int64_t *seg, int64_t p, int64_t T) {
    const int64_t t = p % T;
    return (t == 0 || seg[p] != seg[p - 1]) ? 1 : 0;
}

__global__ void __launch_bounds__(SCAN_THREADS)
    seg_count_kernel(const int64_t *__restrict__ seg, int64_t N, int64_t T, int32_t *tile_sums) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
    int c = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i)
        if (base + i < N) c += seg_flag(seg, base + i, T);
    int total;
    block_exclusive_scan(c, ws, total);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// One CTA: exclusive scan of the tile totals in place; writes the grand
// total to *total_out (if non-null) and to `extra` at index `extra_at` when
// extra is non-null (the cu_seqlens end marker).
__global__ void __launch_bounds__(SCAN_THREADS)
    tile_scan_kernel(int32_t *tile_sums, int64_t n_tiles, int32_t *total_out, int32_t *tail,
                     int32_t tail_value_is_total, int32_t tail_value) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    int carry = 0;
    for (int64_t b0 = 0; b0 < n_tiles; b0 += SCAN_THREADS) {
        const int64_t i = b0 + threadIdx.x;
        const int x = i < n_tiles ? tile_sums[i] : 0;
        int total;
        const int ex = block_exclusive_scan(x, ws, total);
        if (i < n_tiles) tile_sums[i] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) {
        if (total_out) *total_out = carry;
        if (tail) tail[carry] = tail_value_is_total ? carry : tail_value;
    }
}

__global__ void __launch_bounds__(SCAN_THREADS)
    seg_scatter_kernel(const int64_t *__restrict__ seg, int64_t N, int64_t T,
                       const int32_t *__restrict__ tile_offsets, int32_t *__restrict__ cu) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
    int f[SCAN_ITEMS];
    int c = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i) {
        f[i] = (base + i < N) ? seg_flag(seg, base + i, T) : 0;
        c += f[i];
    }
    int total;
    int pos = tile_offsets[blockIdx.x] + block_exclusive_scan(c, ws, total);
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i)
        if (f[i]) cu[pos++] = static_cast<int32_t>(base + i);
}

// ---- prefix sum of lengths (one CTA, no scratch)

__global__ void __launch_bounds__(SCAN_THREADS)
    prefix_sum_kernel(int32_t *__restrict__ cu, const int32_t *__restrict__ len, int64_t n) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    int carry = 0;
    for (int64_t b0 = 0; b0 < n; b0 += SCAN_TILE) {
        const int64_t base = b0 + threadIdx.x * SCAN_ITEMS;
        int x[SCAN_ITEMS];
        int c = 0;
#pragma unroll
        for (int i = 0; i < SCAN_ITEMS; ++i) {
            x[i] = base + i < n ? len[base + i] : 0;
            c += x[i];
        }
        int total;
        int run = carry + block_exclusive_scan(c, ws, total);
#pragma unroll
        for (int i = 0; i < SCAN_ITEMS; ++i) {
            if (base + i < n) cu[base + i] = run;
            run += x[i];
        }
        carry += total;
    }
    if (threadIdx.x == 0) cu[n] = carry;
}

// ---- chunk map

__device__ __forceinline__ int n_chunks_of(const int32_t *cu, int64_t i, int chunk) {
    int len = cu[i + 1] - cu[i];
    return len > 0 ? (len + chunk - 1) / chunk : 0;
}

__global__ void __launch_bounds__(SCAN_THREADS)
    chunk_count_kernel(const int32_t *__restrict__ cu, int64_t n, int chunk, int32_t *tile_sums) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
    int c = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i)
        if (base + i < n) c += n_chunks_of(cu, base + i, chunk);
    int total;
    block_exclusive_scan(c, ws, total);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(SCAN_THREADS)
    chunk_write_kernel(const int32_t *__restrict__ cu, int64_t n, int chunk,
                       const int32_t *__restrict__ tile_offsets, int32_t *__restrict__ chunk_seq,
                       int32_t *__restrict__ chunk_start, int64_t max_chunks) {
    __shared__ int ws[SCAN_THREADS / 32 + 1];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
    int nc[SCAN_ITEMS];
    int c = 0;
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i) {
        nc[i] = base + i < n ? n_chunks_of(cu, base + i, chunk) : 0;
        c += nc[i];
    }
    int total;
    int64_t pos = tile_offsets[blockIdx.x] + block_exclusive_scan(c, ws, total);
#pragma unroll
    for (int i = 0; i < SCAN_ITEMS; ++i) {
        for (int j = 0; j < nc[i]; ++j, ++pos) {
            if (pos < max_chunks) {
                chunk_seq[pos] = static_cast<int32_t>(base + i);
                chunk_start[pos] = cu[base + i] + j * chunk;
            }
        }
    }
}

// ---- state gather / scatter

__global__ void gather_states_kernel(float *__restrict__ dense, const float *__restrict__ pool,
                                     const int32_t *__restrict__ slots, int64_t n,
                                     int64_t num_slots, int H, int64_t dd, bool scatter, bool vec) {
    // One CTA row per (sequence, head); threads stride over the d*d floats.
    for (int64_t item = blockIdx.x; item < n * H; item += gridDim.x) {
        const int64_t i = item / H;
        const int h = static_cast<int>(item - i * H);
        const int64_t slot = slots ? static_cast<int64_t>(slots[i]) : i;
        const bool ok = slot >= 0 && slot < num_slots;
        float *dp = dense + item * dd;
        if (!ok) {
            if (!scatter)
                for (int64_t x = threadIdx.x; x < dd; x += blockDim.x) dp[x] = nanf("");
            continue;
        }
        float *pp = const_cast<float *>(pool) + (slot * H + h) * dd;
        const float *src = scatter ? dp : pp;
        float *dst = scatter ? pp : dp;
        if (vec) {
            const float4 *s4 = reinterpret_cast<const float4 *>(src);
            float4 *d4 = reinterpret_cast<float4 *>(dst);
            for (int64_t x = threadIdx.x; x < dd / 4; x += blockDim.x) d4[x] = s4[x];
        } else {
            for (int64_t x = threadIdx.x; x < dd; x += blockDim.x) dst[x] = src[x];
        }
    }
}

// ---- padded <-> packed token rows

__global__ void pack_tokens_kernel(char *__restrict__ dst, const char *__restrict__ src,
                                   const int32_t *__restrict__ cu, int64_t max_len,
                                   int64_t row_bytes, bool unpack, bool vec16) {
    const int64_t i = blockIdx.y;
    int64_t len = static_cast<int64_t>(cu[i + 1]) - cu[i];
    if (len > max_len) len = max_len;
    if (len < 0) len = 0;
    for (int64_t t = blockIdx.x; t < len; t += gridDim.x) {
        const int64_t prow = cu[i] + t;
        const int64_t qrow = i * max_len + t;
        const char *s = src + (unpack ? prow : qrow) * row_bytes;
        char *d = dst + (unpack ? qrow : prow) * row_bytes;
        if (vec16) {
            for (int64_t x = threadIdx.x; x < row_bytes / 16; x += blockDim.x)
                reinterpret_cast<int4 *>(d)[x] = reinterpret_cast<const int4 *>(s)[x];
        } else {
            for (int64_t x = threadIdx.x; x < row_bytes / 4; x += blockDim.x)
                reinterpret_cast<int32_t *>(d)[x] = reinterpret_cast<const int32_t *>(s)[x];
        }
    }
}

// ---- head-sharded outputs: rank-major gather buffer <-> [tokens][H][d]

// out[tok][r * Hs + hh][:] = gathered[r][tok][hh][:] (unshard), or the
// reverse (shard), for rows of row_bytes; one CTA row loop per (r, tok).
__global__ void heads_unshard_kernel(char *__restrict__ dst, const char *__restrict__ src,
                                     int64_t G, int64_t tokens, int64_t Hs, int64_t row_bytes,
                                     bool shard, bool vec16) {
    const int64_t slab = Hs * row_bytes;  // one rank's rows of one token
    for (int64_t u = blockIdx.x; u < G * tokens; u += gridDim.x) {
        const int64_t r = u / tokens, tok = u - r * tokens;
        const int64_t goff = (r * tokens + tok) * slab;           // gathered layout
        const int64_t ooff = (tok * G + r) * slab;                // [tok][r][Hs][d] == [tok][H][d]
        const char *s = src + (shard ? ooff : goff);
        char *d = dst + (shard ? goff : ooff);
        if (vec16) {
            for (int64_t x = threadIdx.x; x < slab / 16; x += blockDim.x)
                reinterpret_cast<int4 *>(d)[x] = reinterpret_cast<const int4 *>(s)[x];
        } else {
            for (int64_t x = threadIdx.x; x < slab / 4; x += blockDim.x)
                reinterpret_cast<int32_t *>(d)[x] = reinterpret_cast<const int32_t *>(s)[x];
        }
    }
}

int64_t tiles_of(int64_t n) { return (n + SCAN_TILE - 1) / SCAN_TILE; }

}  // namespace

size_t varlen_ws_bytes(int64_t n) {
    const int64_t tiles = tiles_of(n > 0 ? n : 1);
    return static_cast<size_t>((tiles * 4 + 255) / 256 * 256);
}

int launch_prefix_sum(int32_t *cu, const int32_t *lengths, int64_t n, cudaStream_t s) {
    prefix_sum_kernel<<<1, SCAN_THREADS, 0, s>>>(cu, lengths, n);
    return check_launch("prefix_sum_kernel");
}

int launch_segments_to_cu(int32_t *cu, int32_t *n_seg, const int64_t *segment, int64_t B,
                          int64_t T, void *ws, size_t ws_bytes, cudaStream_t s) {
    const int64_t N = B * T;
    const int64_t tiles = tiles_of(N);
    if (ws_bytes < varlen_ws_bytes(N) || ws == nullptr)
        return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu",
                         varlen_ws_bytes(N), ws_bytes);
    int32_t *tile_sums = static_cast<int32_t *>(ws);
    if (N == 0) {
        cudaMemsetAsync(cu, 0, sizeof(int32_t), s);
        cudaMemsetAsync(n_seg, 0, sizeof(int32_t), s);
        return check_launch("segments_to_cu (empty)");
    }
    seg_count_kernel<<<static_cast<unsigned>(tiles), SCAN_THREADS, 0, s>>>(segment, N, T, tile_sums);
    tile_scan_kernel<<<1, SCAN_THREADS, 0, s>>>(tile_sums, tiles, n_seg, cu, 0,
                                                static_cast<int32_t>(N));
    seg_scatter_kernel<<<static_cast<unsigned>(tiles), SCAN_THREADS, 0, s>>>(segment, N, T, tile_sums, cu);
    return check_launch("segments_to_cu");
}

int launch_chunk_map(int32_t *chunk_seq, int32_t *chunk_start, int32_t *n_chunks,
                     const int32_t *cu, int64_t n_seq, int chunk, int64_t max_chunks, void *ws,
                     size_t ws_bytes, cudaStream_t s) {
    const int64_t tiles = tiles_of(n_seq);
    if (ws_bytes < varlen_ws_bytes(n_seq) || ws == nullptr)
        return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu",
                         varlen_ws_bytes(n_seq), ws_bytes);
    if (n_seq == 0) {
        cudaMemsetAsync(n_chunks, 0, sizeof(int32_t), s);
        return check_launch("chunk_map (empty)");
    }
    int32_t *tile_sums = static_cast<int32_t *>(ws);
    chunk_count_kernel<<<static_cast<unsigned>(tiles), SCAN_THREADS, 0, s>>>(cu, n_seq, chunk, tile_sums);
    tile_scan_kernel<<<1, SCAN_THREADS, 0, s>>>(tile_sums, tiles, n_chunks, nullptr, 0, 0);
    chunk_write_kernel<<<static_cast<unsigned>(tiles), SCAN_THREADS, 0, s>>>(
        cu, n_seq, chunk, tile_sums, chunk_seq, chunk_start, max_chunks);
    return check_launch("chunk_map");
}

int launch_gather_states(float *dense, const float *pool, const int32_t *slots, int64_t n,
                         int64_t num_slots, int H, int d, bool scatter, cudaStream_t s) {
    if (n == 0) return RHZ_OK;
    const int64_t dd = static_cast<int64_t>(d) * d;
    const bool vec = (dd % 4) == 0 && aligned(dense, 16) && aligned(pool, 16);
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    int64_t grid = n * H;
    if (grid > static_cast<int64_t>(sms) * 32) grid = static_cast<int64_t>(sms) * 32;
    gather_states_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(dense, pool, slots, n,
                                                                      num_slots, H, dd, scatter, vec);
    return check_launch(scatter ? "scatter_states" : "gather_states");
}

int launch_heads_unshard(void *dst, const void *src, int64_t G, int64_t tokens, int64_t Hs,
                         int64_t row_bytes, bool shard, cudaStream_t s) {
    if (G == 0 || tokens == 0 || Hs == 0 || row_bytes == 0) return RHZ_OK;
    const int64_t slab = Hs * row_bytes;
    const bool vec16 = slab % 16 == 0 && aligned(dst, 16) && aligned(src, 16);
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    int64_t grid = G * tokens;
    if (grid > static_cast<int64_t>(sms) * 16) grid = static_cast<int64_t>(sms) * 16;
    int threads = static_cast<int>(slab / (vec16 ? 16 : 4));
    threads = threads < 32 ? 32 : (threads > 256 ? 256 : (threads + 31) / 32 * 32);
    heads_unshard_kernel<<<static_cast<unsigned>(grid), threads, 0, s>>>(
        static_cast<char *>(dst), static_cast<const char *>(src), G, tokens, Hs, row_bytes, shard,
        vec16);
    return check_launch(shard ? "heads_shard" : "heads_unshard");
}

int launch_pack_tokens(void *dst, const void *src, const int32_t *cu, int64_t n, int64_t max_len,
                       int64_t row_bytes, bool unpack, cudaStream_t s) {
    if (n == 0 || max_len == 0 || row_bytes == 0) return RHZ_OK;
    const bool vec16 = row_bytes % 16 == 0 && aligned(dst, 16) && aligned(src, 16);
    int64_t gx = max_len < 1024 ? max_len : 1024;
    int threads = static_cast<int>(row_bytes / (vec16 ? 16 : 4));
    threads = threads < 32 ? 32 : (threads > 256 ? 256 : (threads + 31) / 32 * 32);
    if (n > 65535) return set_error(RHZ_ERR_SHAPE, "pack_tokens: n = %lld > 65535 sequences", (long long)n);
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(n));
    pack_tokens_kernel<<<grid, threads, 0, s>>>(static_cast<char *>(dst),
                                                static_cast<const char *>(src), cu, max_len,
                                                row_bytes, unpack, vec16);
    return check_launch(unpack ? "unpack_tokens" : "pack_tokens");
}

// ---------------------------------------------------------------- no-allocation variant
//
// rhz_varlen_segments_to_cu_seqlens_noalloc keeps the scan's per-tile totals
// (its only scratch) in a file-scope device array instead of a caller
// workspace, for callers that have no way to allocate device memory (see the
// header). Limit: RHZ_NOALLOC_MAX_POSITIONS = 2^26 positions, i.e. 16384
// tiles of 4096 -> 64 KiB per GPU, held from library load until process exit.
// Every call shares this one array and it keeps the last call's contents;
// nothing needs clearing because each call writes every tile total it reads
// before reading it. Calls whose kernels overlap on the GPU (different
// streams, or different host threads on the same device) race on it.

namespace {
constexpr int64_t NOALLOC_TILES = RHZ_NOALLOC_MAX_POSITIONS / SCAN_TILE;
static_assert(NOALLOC_TILES * SCAN_TILE == RHZ_NOALLOC_MAX_POSITIONS, "limit is a whole number of tiles");
}  // namespace

static __device__ __align__(256) int32_t g_noalloc_tile_sums[NOALLOC_TILES];

namespace {

// Device address of g_noalloc_tile_sums on the current device. The name is a
// host-side stand-in, not a device address, so it is resolved with
// cudaGetSymbolAddress once per device (with that device current) and cached.
struct NoallocScratch {
    std::mutex mu;
    int32_t *ptr = nullptr;
};
NoallocScratch g_noalloc[64];

int noalloc_scratch(int32_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(RHZ_ERR_DEVICE, "device ordinal %d out of range", dev);
    NoallocScratch &s = g_noalloc[dev];
    std::lock_guard<std::mutex> lock(s.mu);
    if (s.ptr == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_tile_sums);
        if (e != cudaSuccess)
            return set_error(RHZ_ERR_DEVICE, "cudaGetSymbolAddress(no-allocation scratch): %s",
                             cudaGetErrorString(e));
        s.ptr = static_cast<int32_t *>(p);
    }
    *out = s.ptr;
    return RHZ_OK;
}

}  // namespace
}  // namespace rhz

extern "C" int rhz_varlen_segments_to_cu_seqlens_noalloc(int32_t *cu_seqlens, int32_t *n_seg_out,
                                                         const int64_t *segment, int64_t B,
                                                         int64_t T, rhz_stream_t stream) {
    using namespace rhz;
    clear_error();
    if (B < 0 || T < 0)
        return set_error(RHZ_ERR_SHAPE, "B = %lld, T = %lld: must be >= 0", (long long)B, (long long)T);
    if (T > 0 && B > RHZ_NOALLOC_MAX_POSITIONS / T)
        return set_error(RHZ_ERR_SHAPE,
                         "B*T = %lld x %lld exceeds the no-allocation limit of %lld positions; "
                         "use rhz_varlen_segments_to_cu_seqlens with a workspace",
                         (long long)B, (long long)T, (long long)RHZ_NOALLOC_MAX_POSITIONS);
    if (cu_seqlens == nullptr || n_seg_out == nullptr || !aligned(cu_seqlens, 4) || !aligned(n_seg_out, 4))
        return set_error(RHZ_ERR_INVALID, "cu_seqlens / n_seg_out must be non-NULL int32 pointers");
    if (B * T > 0 && (segment == nullptr || !aligned(segment, 8)))
        return set_error(RHZ_ERR_INVALID, "segment must be a non-NULL 8-byte aligned int64 pointer");
    int sms = 0;
    bool sm100 = false;
    int st = device_info(&sms, &sm100);
    if (st != RHZ_OK) return st;
    if (!sm100) return set_error(RHZ_ERR_DEVICE, "this library is built for sm_100a (B200) only");
    int32_t *scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != RHZ_OK) return st;
    return launch_segments_to_cu(cu_seqlens, n_seg_out, segment, B, T, scratch,
                                 static_cast<size_t>(NOALLOC_TILES) * sizeof(int32_t),
                                 as_cuda(stream));
}
