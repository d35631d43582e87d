// Shared device helpers for the B200 sampler kernels.
//
// Exactness rules used everywhere a value can reach the sampled token: each
// fp32 operation of the reference (sampler.h) is issued as the matching
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, ...) so that
// nvcc cannot contract a multiply and an add into one FMA, and the library is
// built with --fmad=false as a second guard.  expf is CUDA's accurate expf
// (never __expf / fast-math).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qs_exp.cuh"
#include "qwen600_sampler.h"

namespace qs {

using qs_row_debug_dev = ::qs_row_debug;

constexpr int kThreads = 512;          // threads per row CTA
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVocab = 262144;      // fast-kernel limit (segment tables in smem)
constexpr int kCandCap = 2048;         // candidate buffer of the row kernel
constexpr int kMaxWindow = 2048;       // penalty window limit
constexpr float kSigGap = 17.5f;       // e^-17.5 < 2^-25 with margin: below it a term
                                       // cannot change a running fp32 sum >= e^(gap)

// Launch parameters of the row and exact-tie kernels.
struct RowParams {
    float temperature, topp, minp;
    int top_k;
    unsigned flags;
};
constexpr int kStashCap = 1536;  // stashed elements per row before the dense method

// What the row kernel's streaming pass leaves for its finishing pass, per row
// (global memory): the penalised segment maxima.
// Where a vocabulary-sharded launch stores its logits: batch row b (of the
// call, counted from row0) belongs to rank (row0 + b) / rows_per and goes to
// row (row0 + b) % rows_per of that rank's [rows_per, ld] buffer, at column
// col0 + the tile's column.  nranks == 0: the plain [B, V] output.
constexpr int kLhMaxRanks = 8;
struct LhPeer {
    __nv_bfloat16* dst[kLhMaxRanks];
    int nranks, rows_per, row0, col0;
    long long ld;
};

struct RowScratch {
    float* segm;               // [rows][seg_stride] penalised segment maxima (scan -> gather, finish)
    int seg_stride;
    int* done;                 // [rows] greedy: chunks scanned; the last one finishes the row and
                               // clears done and gmax for the next call
    unsigned long long* gmax;  // [rows] greedy: packed (order key, ~index) of the largest
                               // penalised logit so far
    int2* stash;               // [rows][stash_cap] (index, t bits): the rows' significant elements
    int stash_cap;
    int* stash_used;           // [rows] entries claimed (the finish clears it)
    int* chunk_off;            // [rows][max_chunks] where each chunk's run starts (-1: none)
    int* chunk_n;              // [rows][max_chunks] its length (-1: overflowed)
    float* chunk_lb;           // [rows][max_chunks] the largest significance bound it used
    int max_chunks;
    // dense rows: the exact terms of the hot segments whose running-sum binade
    // cannot be predicted, formed in parallel before the sequential walk
    float* fb_terms;           // [fb_rows][kFbCap][256]
    int fb_rows;               // rows it has room for (0: none; the walk forms them itself)
    // bf16 rows whose producer already formed the segment maxima (the lm_head
    // epilogue): order keys (fkey) of the raw maxima of the full 256-element
    // segments, [rows][premax_stride]; the scan reads them instead of
    // streaming the row and leaves the buffer zeroed.  nullptr: stream.
    uint32_t* premax;
    int premax_stride;
};
constexpr int kFbCap = 64;      // segments per row with precomputed exact terms
// Segment maxima per row that fit either element type (fp32 segments are the
// shorter: 128 elements).
inline int row_scratch_seg_stride(int V) { return (V + 127) / 128; }
constexpr int kRowChunkSegs = 64;  // segments per chunk scan (one CTA each)
inline int row_chunks(int V, int seg) { return ((V + seg - 1) / seg + kRowChunkSegs - 1) / kRowChunkSegs; }
inline int row_max_chunks(int V) { return row_chunks(V, 128); }  // the shorter (fp32) segments

struct TieParams {
    float temperature, topp, minp;
    int top_k;
};

// The row's penalty window and the override tables the row kernel writes
// for the later passes (ties, probabilities, penalised write-back).
struct RowWindow {
    const int* hist;          // [B, window] token ids (slot order), or NULL
    const int* count;         // [B] slots in use
    const float* slot_counts; // [B, window] count of each slot's token, or NULL
    int window;
    float rp, fp, pp;
    int* ov_n;                // [B] out: distinct in-range window tokens
    int* ov_idx;              // [B, ov_stride] out: those tokens, ascending
    float* ov_val;            // [B, ov_stride] out: their penalised logits
    int ov_stride;
};

// Per-row results shared between the row kernel, the exact-tie kernel, the
// history update and the debug readers.  Mirrors qs_row_debug's first fields.
struct RowResult {
    int token;
    int greedy;
    int n_topk;
    int n_minp;
    int n_final;
    int draw_pos;
    int exact_ties;
    int sum_fallback;
    float max_logit;
    float sum;
    float r;
    float renorm_sum;
    // internals for the exact-tie pass
    float inv_temp;
    float sum_inv;
    int status;      // 0 ok, >0 unsupported input for the fast kernel
    int pad_;
};

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
    static constexpr int kPerLane = 4;  // one 16-byte load per lane
    __device__ __forceinline__ static float widen(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int kPerLane = 8;
    __device__ __forceinline__ static float widen(__nv_bfloat16 v) { return __bfloat162float(v); }
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out);

template <>
__device__ __forceinline__ void load_vec<float>(const float* p, float* out) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}

template <>
__device__ __forceinline__ void load_vec<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// --------------------------------------------------------------- keys
// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey_bits(uint32_t u) {
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t fkey(float f) { return fkey_bits(__float_as_uint(f)); }
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// Maximum of one 16-byte vector of logits (a lane's share of a segment; bf16
// pairs compared packed).  The streaming passes and the lm_head epilogue form
// segment maxima with it, so both give the same bits.
template <typename T>
__device__ __forceinline__ float vec_max(const uint4& r);
template <>
__device__ __forceinline__ float vec_max<__nv_bfloat16>(const uint4& r) {
    __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
    __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&r.z);
    __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&r.w);
    __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return fmaxf(__low2float(m), __high2float(m));
}
template <>
__device__ __forceinline__ float vec_max<float>(const uint4& r) {
    return fmaxf(fmaxf(__uint_as_float(r.x), __uint_as_float(r.y)),
                 fmaxf(__uint_as_float(r.z), __uint_as_float(r.w)));
}

// ------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_min_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide reductions for kThreads threads; `red` holds >= kWarps slots.
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = lane < kWarps ? red[lane] : -INFINITY;
    return warp_max(r);
}
__device__ __forceinline__ int block_min_int(int v, int* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_min_int(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int r = lane < kWarps ? red[lane] : 0x7fffffff;
    return warp_min_int(r);
}
__device__ __forceinline__ int block_sum_int(int v, int* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum_int(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int r = lane < kWarps ? red[lane] : 0;
    return warp_sum_int(r);
}

// Exclusive prefix sum of one int per thread across the block; returns the
// block total in *total.
__device__ __forceinline__ int block_excl_scan_int(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = lane < kWarps ? red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kWarps) red[lane] = s;  // inclusive per-warp totals
    }
    __syncthreads();
    int before = (w == 0) ? 0 : red[w - 1];
    *total = red[kWarps - 1];
    return before + x - v;
}

// ------------------------------------------------------------- RNG
// xorshift64* (sampler.h:49-60): shifts 12/25/27, multiplier
// 0x2545F4914F6CDD1D, high 32 bits of the product; the uniform keeps 24 bits.
__device__ __forceinline__ float xorshift_f32(unsigned long long* st) {
    unsigned long long x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    uint32_t u = (uint32_t)((x * 0x2545F4914F6CDD1Dull) >> 32);
    return __fmul_rn((float)(u >> 8), 5.9604644775390625e-08f);  // exact /2^24
}

}  // namespace qs
