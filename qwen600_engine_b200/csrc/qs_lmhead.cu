// The decode step's tail before sampling: the final RMSNorm and the lm_head
// projection (qwen_model.cuh:710-723), on sm_100a.
//
// rmsnorm_rows_kernel restates rms_norm_kernel (qwen_model.cuh:125-177) row
// by row: per-thread fma chains over bf16 pairs, a 256-thread cub block sum,
// mul = rsqrtf(fma(sum, 1/D, eps)), y = bf16((x * mul) * w).  The reference
// normalises one row per call; here a CTA per row of the batch.
//
// lm_head_kernel computes logits[B, V] = bf16(normed[B, K] . W[V, K]^T) with
// fp32 accumulation, as the reference's cublasGemmEx call does
// (qwen_model.cuh:607-629: bf16 inputs and output, fp32 compute).  It is a
// persistent, warp-specialised tcgen05 GEMM:
//   warp 0  one thread issues TMA loads (128B-swizzled K-major tiles of the
//           normed hidden rows and of N vocabulary rows of W) into a
//           4-stage shared-memory ring;
//   warp 1  one thread issues tcgen05.mma (M = 128 batch rows, N = 128..208
//           vocabulary rows, K = 16 per instruction) into one of two TMEM
//           accumulators, and tcgen05.commit frees each stage and hands
//           a finished accumulator to the epilogue;
//   warps 2-5 read the accumulator with tcgen05.ld (each warp its 32 TMEM
//           lanes = 32 batch rows), round to bf16 and store the logits:
//           to [B, V], or, for a vocabulary-sharded launch, each row to the
//           buffer of the GPU that samples it (bulk copies over NVLink).
// W is read from HBM exactly once per launch (311 MB for Qwen3-0.6B: the
// bound); the hidden rows (at most 256 KB) are re-read from L2 per tile.
// Every wait is bounded: after kLhWaitNs the kernel raises an error flag,
// lets the copies and MMAs it issued finish, frees its TMEM and returns.
#include <cuda.h>
#include <string.h>
#include <cudaTypedefs.h>

#include <cub/block/block_reduce.cuh>

#include "qs_common.cuh"
#include "qs_pipe.cuh"

namespace qs {

constexpr int kLhM = 128;                       // batch rows per launch (MMA M)
constexpr int kLhK = 64;                        // K per stage: one 128-byte swizzle row
constexpr int kLhStages = 4;
constexpr int kLhThreads = 192;
constexpr uint32_t kLhStageA = kLhM * kLhK * 2;  // 16 KB
constexpr uint32_t kLhAccStride = 256;           // TMEM columns between the two accumulators
constexpr uint32_t kLhTmemCols = 2 * kLhAccStride;
constexpr unsigned long long kLhWaitNs = 2000000000ull;

struct LhShared {
    unsigned long long full[kLhStages];
    unsigned long long empty[kLhStages];
    unsigned long long tfull[2];
    unsigned long long tempty[2];
    uint32_t tmem_base;
    int abort;
};

// Vocabulary rows per tile (MMA N, a multiple of 16 up to 256), chosen per
// launch so the tiles spread evenly over the SMs: 208 for Qwen3's 151,936
// rows on one GPU (731 tiles over 148 SMs within 1.2% of evenly), narrower
// tiles for the slices of a vocabulary-sharded launch.
template <int N>
struct LhTile {
    static_assert(N % 16 == 0 && N >= 16 && N <= 256, "MMA N");
    static constexpr uint32_t kStageB = N * kLhK * 2;
    static constexpr uint32_t kOutTile = 32 * N * 2;  // one epilogue warp's bf16 rows of a tile
    // tcgen05.mma kind::f16 instruction descriptor: fp32 accumulator, bf16 A
    // and B, both K-major, N, M = 128.
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                                       ((uint32_t)(kLhM >> 4) << 24);
    static size_t smem() {
        return 1024 + kLhStages * (size_t)(kLhStageA + kStageB) + 4 * (size_t)kOutTile + sizeof(LhShared);
    }
};

constexpr unsigned long long kLhDrainNs = 100000000ull;  // 100 ms
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, unsigned long long* bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"((unsigned long long)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile whose
// rows are 128 bytes apart (8-row groups 1024 bytes apart).
__device__ __forceinline__ unsigned long long sw128_desc(uint32_t saddr) {
    return (unsigned long long)((saddr >> 4) & 0x3FFFu)  // start address
           | (1ull << 16)                                 // leading byte offset (16 B)
           | (64ull << 32)                                // stride byte offset (1024 B)
           | (1ull << 46)                                 // descriptor version (sm_100)
           | (2ull << 61);                                // 128-byte swizzle
}
__device__ __forceinline__ void umma_bf16(uint32_t dtmem, unsigned long long adesc, unsigned long long bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int N>
__global__ void __launch_bounds__(kLhThreads, 1)
lm_head_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, int tma_out, __nv_bfloat16* __restrict__ out, int B,
               int V, int K, int ntiles, int* __restrict__ err, const __grid_constant__ LhPeer peer,
               unsigned long long wait_ns, uint32_t* __restrict__ segk, int segk_stride) {
    using Tl = LhTile<N>;
    constexpr uint32_t kLhStageB = Tl::kStageB;
    constexpr uint32_t kLhOutTile = Tl::kOutTile;
    constexpr int kLhN = N;
    extern __shared__ unsigned char lh_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(lh_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* sA = base;                              // [stages][128 x 64 bf16]
    unsigned char* sB = base + kLhStages * kLhStageA;      // [stages][kLhN x 64 bf16]
    unsigned char* sC = sB + kLhStages * kLhStageB;          // [4 warps][32 x kLhN bf16]
    LhShared* sh = reinterpret_cast<LhShared*>(sC + 4 * kLhOutTile);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = K / kLhK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLhStages; s++) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sh->tfull[b], 1);
            mbar_init(&sh->tempty[b], 4);  // one arrival per epilogue warp
        }
        sh->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&tmB) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sh->tmem_base)),
                     "r"(kLhTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sh->tmem_base;
    volatile int* abort = &sh->abort;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer
            int s = 0;
            uint32_t ph = 0;
            int last_ph[kLhStages];
            for (int i = 0; i < kLhStages; i++) last_ph[i] = -1;
            bool stop = false;
            // launched as a programmatic dependent of the RMSNorm kernel: the
            // set-up above overlaps it; its rows are read only after it ends
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x) {
                for (int kb = 0; kb < nk; kb++) {
                    if (!mbar_wait(&sh->empty[s], ph ^ 1u, abort, wait_ns)) { stop = true; break; }
                    mbar_expect_tx(&sh->full[s], kLhStageA + kLhStageB);
                    tma_load_2d(sA + s * kLhStageA, &tmA, &sh->full[s], kb * kLhK, 0);
                    tma_load_2d(sB + s * kLhStageB, &tmB, &sh->full[s], kb * kLhK, tile * kLhN);
                    last_ph[s] = (int)ph;
                    if (++s == kLhStages) { s = 0; ph ^= 1u; }
                }
            }
            if (*abort) {
                // let the copies this thread issued land before the CTA leaves
                for (int i = 0; i < kLhStages; i++)
                    if (last_ph[i] >= 0) mbar_wait(&sh->full[i], (uint32_t)last_ph[i], abort, kLhDrainNs, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            int s = 0;
            uint32_t ph = 0;
            unsigned long long* last_bar = nullptr;
            uint32_t last_par = 0;
            bool stop = false;
            int it = 0;
            for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x, it++) {
                const int b = it & 1;
                const uint32_t use = (uint32_t)(it >> 1);
                if (!mbar_wait(&sh->tempty[b], (use & 1u) ^ 1u, abort, wait_ns)) break;
                tc_fence_after();
                const uint32_t dt = tbase + (uint32_t)b * kLhAccStride;
                for (int kb = 0; kb < nk; kb++) {
                    if (!mbar_wait(&sh->full[s], ph, abort, wait_ns)) { stop = true; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * kLhStageA);
                    const uint32_t b0 = smem_u32(sB + s * kLhStageB);
#pragma unroll
                    for (int kk = 0; kk < kLhK / 16; kk++)
                        umma_bf16(dt, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), Tl::kIdesc,
                                  (kb | kk) != 0 ? 1u : 0u);
                    umma_commit(&sh->empty[s]);
                    last_bar = &sh->empty[s];
                    last_par = ph;
                    if (++s == kLhStages) { s = 0; ph ^= 1u; }
                }
                if (stop) break;
                umma_commit(&sh->tfull[b]);
                last_bar = &sh->tfull[b];
                last_par = use & 1u;
            }
            if (*abort && last_bar)  // the MMAs and commits issued complete before TMEM is freed
                mbar_wait(last_bar, last_par, abort, kLhDrainNs, false);
        }
    } else {
        // ---- epilogue: warps 2..5, each on its quarter of the TMEM lanes
        // (32 batch rows).  With tma_out the warp stages its rows of the tile
        // in shared memory and one lane stores them with a TMA bulk tensor
        // copy (whole row segments; rows past B and columns past V are
        // clipped by the copy).  In a sharded launch (peer.nranks > 0) the
        // warp stages its rows the same way and each lane copies its row
        // segment to the buffer of the rank that samples that row (this
        // GPU's or a peer's over NVLink) with one bulk copy.  Otherwise each
        // lane stores its own row.
        const bool staged = tma_out || peer.nranks > 0;
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const bool vec = (V % 8) == 0;
        __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(sC + q * kLhOutTile) + lane * kLhN;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, it++) {
            const int b = it & 1;
            const uint32_t use = (uint32_t)(it >> 1);
            if (!mbar_wait(&sh->tfull[b], use & 1u, abort, wait_ns)) break;
            tc_fence_after();
            const int n0 = tile * kLhN;
            if (tma_out && lane == 0)  // the previous tile's store has read the staging rows
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            if (peer.nranks > 0)  // this lane's previous row copy has read its staging row
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
            // the row's running segment maximum (order key) over this tile's
            // columns; 16-column pieces never straddle a 256-column segment
            uint32_t run = 0u;
            int rseg = n0 >> 8;
#pragma unroll 1
            for (int c = 0; c < kLhN / 16; c++) {
                uint32_t r[16];
                tmem_ld16(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)b * kLhAccStride + (uint32_t)(c * 16), r);
                uint32_t pk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]),
                                                                  __uint_as_float(r[2 * j + 1]));
                    pk[j] = *reinterpret_cast<const uint32_t*>(&h);
                }
                if (segk && n0 + c * 16 < V) {
                    const int sg = (n0 + c * 16) >> 8;
                    if (sg != rseg) {
                        if (run && row < B) atomicMax(segk + (size_t)row * segk_stride + rseg, run);
                        run = 0u;
                        rseg = sg;
                    }
                    if (n0 + c * 16 + 16 <= V) {
                        // per 8 columns, as a streaming lane forms them
                        const uint32_t k1 = fkey(vec_max<__nv_bfloat16>(make_uint4(pk[0], pk[1], pk[2], pk[3])));
                        const uint32_t k2 = fkey(vec_max<__nv_bfloat16>(make_uint4(pk[4], pk[5], pk[6], pk[7])));
                        run = max(run, max(k1, k2));
                    }
                }
                if (staged) {
                    uint4* d4 = reinterpret_cast<uint4*>(stage + c * 16);
                    d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    continue;
                }
                const int col = n0 + c * 16;
                if (row < B && col < V) {
                    __nv_bfloat16* dst = out + (size_t)row * V + col;
                    if (vec && col + 16 <= V) {
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
                        d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    } else {
                        for (int j = 0; j < 16 && col + j < V; j++)
                            dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
                    }
                }
            }
            if (run && row < B) atomicMax(segk + (size_t)row * segk_stride + rseg, run);
            tc_fence_before();
            if (staged) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sh->tempty[b]);
                if (tma_out) {
                    asm volatile(
                        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                            (unsigned long long)&tmC),
                        "r"(n0), "r"(q * 32), "r"(smem_u32(sC + q * kLhOutTile))
                        : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            // (the accumulator is released above: its values are in the staging rows)
            if (peer.nranks > 0 && row < B) {
                // each lane's row segment to the rank that samples the row, as
                // one bulk copy (over NVLink for a peer; 16-byte aligned: the
                // host checks the buffers, col0 and the vocabulary)
                const int grow = peer.row0 + row;
                const int rk = grow / peer.rows_per;
                const int ncols = min(kLhN, V - n0);
                __nv_bfloat16* d = peer.dst[rk] + (size_t)(grow - rk * peer.rows_per) * peer.ld + peer.col0 + n0;
                asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(d),
                             "r"(smem_u32(stage)), "r"(ncols * 2)
                             : "memory");
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
        }
        if (tma_out && lane == 0)  // the last stores complete before the CTA leaves
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        if (peer.nranks > 0) {
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // this lane's row copies are done
            __threadfence_system();  // and visible to the peers before the kernel ends
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kLhTmemCols)
                     : "memory");
    }
    if (threadIdx.x == 0 && *abort) atomicExch(err, 1);
}

// Completion handshake of a vocabulary-sharded launch, on the stream after
// it: lane r publishes `epoch` into rank r's flag word for this rank
// (release, system scope: this GPU's peer stores of the launch before it are
// visible first), then waits until rank r's word in this rank's flags
// reaches `epoch` (acquire).  The wait is bounded by limit_ns; then *err = 1
// and the lane returns.  Flags: nranks words at byte offset flag_off of every
// rank's buffer, word s written by rank s.
struct ShardFlags {
    unsigned char* base[kLhMaxRanks];
};
__global__ void shard_handshake_kernel(const __grid_constant__ ShardFlags f, size_t flag_off, int nranks,
                                       int rank, unsigned epoch, unsigned long long limit_ns,
                                       int* __restrict__ err) {
    const int r = threadIdx.x;
    if (r >= nranks) return;
    __threadfence_system();
    unsigned* dst = reinterpret_cast<unsigned*>(f.base[r] + flag_off) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const unsigned* mine = reinterpret_cast<const unsigned*>(f.base[rank] + flag_off) + r;
    const unsigned long long t0 = global_ns();
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if ((int)(v - epoch) >= 0) break;
        if (global_ns() - t0 > limit_ns) {
            atomicExch(err, 1);
            break;
        }
    }
}

cudaError_t launch_shard_handshake(void* const* bufs, size_t flag_off, int nranks, int rank, unsigned epoch,
                                   unsigned long long limit_ns, int* err, cudaStream_t stream) {
    ShardFlags f;
    memset(&f, 0, sizeof(f));
    for (int r = 0; r < nranks; r++) f.base[r] = static_cast<unsigned char*>(bufs[r]);
    shard_handshake_kernel<<<1, 32, 0, stream>>>(f, flag_off, nranks, rank, epoch, limit_ns, err);
    return cudaGetLastError();
}

// Restates rms_norm_kernel (qwen_model.cuh:125-177) for one row per CTA.
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ w,
                    __nv_bfloat16* __restrict__ Y, int D, float inv_d, float eps) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the lm_head may start its set-up
    const int t = threadIdx.x;
    const int half = D / 2;
    const __nv_bfloat162* in = reinterpret_cast<const __nv_bfloat162*>(X + (size_t)blockIdx.x * D);
    const __nv_bfloat162* wt = reinterpret_cast<const __nv_bfloat162*>(w);
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(Y + (size_t)blockIdx.x * D);
    float lsum = 0.0f;
    for (int i = t; i < half; i += kNormThreads) {
        const float2 v = __bfloat1622float2(in[i]);
        lsum = __fmaf_rn(v.x, v.x, lsum);
        lsum = __fmaf_rn(v.y, v.y, lsum);
    }
    using BlockReduce = cub::BlockReduce<float, kNormThreads>;
    __shared__ typename BlockReduce::TempStorage tmp;
    const float total = BlockReduce(tmp).Sum(lsum);
    __shared__ float mul;
    if (t == 0) mul = rsqrtf(__fmaf_rn(total, inv_d, eps));
    __syncthreads();
    const float m = mul;
    for (int i = t; i < half; i += kNormThreads) {
        float2 v = __bfloat1622float2(in[i]);
        const float2 g = wt ? __bfloat1622float2(wt[i]) : make_float2(1.0f, 1.0f);
        v.x = __fmul_rn(__fmul_rn(v.x, m), g.x);
        v.y = __fmul_rn(__fmul_rn(v.y, m), g.y);
        o[i] = __float22bfloat162_rn(v);
    }
}

// ------------------------------------------------------------- host side
// The time limit of the kernel's pipeline waits; lm_head_set_wait_ns lets a
// test make them run out (0 restores the default).
static unsigned long long g_wait_ns = kLhWaitNs;
void lm_head_set_wait_ns(unsigned long long ns) { g_wait_ns = ns ? ns : kLhWaitNs; }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// A [rows, K] bf16 row-major matrix as 128B-swizzled [box_rows x 64] tiles.
static bool make_map(CUtensorMap* m, const void* ptr, int rows, int K, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kLhK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int N>
static cudaError_t lm_head_go(const CUtensorMap& ma, const __nv_bfloat16* W, __nv_bfloat16* logits, int B,
                              int V, int K, int num_sms, int* err, const LhPeer& peer, uint32_t* segk,
                              int segk_stride, cudaStream_t stream) {
    CUtensorMap mb;
    if (!make_map(&mb, W, V, K, N)) return cudaErrorInvalidValue;
    // the logits as [B, V] with 32-row x N-column boxes, unswizzled (row
    // pitch V * 2 bytes must be a multiple of 16)
    CUtensorMap mc;
    memset(&mc, 0, sizeof(mc));
    int tma_out = 0;
    if (peer.nranks == 0 && (V % 8) == 0 && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0)) {
        auto fn = encode_fn();
        const cuuint64_t dims[2] = {(cuuint64_t)V, (cuuint64_t)B};
        const cuuint64_t strides[1] = {(cuuint64_t)V * 2};
        const cuuint32_t box[2] = {(cuuint32_t)N, 32};
        const cuuint32_t estr[2] = {1, 1};
        tma_out = fn && fn(&mc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, logits, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    const int ntiles = (V + N - 1) / N;
    const int grid = ntiles < num_sms ? ntiles : num_sms;
    const size_t smem = LhTile<N>::smem();
    cudaError_t e = cudaFuncSetAttribute(lm_head_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: the kernel may start while the launch
    // before it (the RMSNorm) runs, and waits for it before its first load
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLhThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lm_head_kernel<N>, ma, mb, mc, tma_out, logits, B, V, K, ntiles, err, peer,
                              g_wait_ns, segk, segk_stride);
}

// The tile width whose tiles spread most evenly over num_sms persistent CTAs
// (time ~ waves x N); ties go to the wider tile.
int lm_head_tile(int V, int num_sms) {
    static const int cand[] = {208, 176, 144, 128};
    int best = cand[0];
    long long best_cost = -1;
    for (int n : cand) {
        const long long tiles = (V + n - 1) / n;
        const long long cost = ((tiles + num_sms - 1) / num_sms) * n;
        if (best_cost < 0 || cost < best_cost) { best = n; best_cost = cost; }
    }
    return best;
}

static cudaError_t lm_head_dispatch(const __nv_bfloat16* normed, const __nv_bfloat16* W, __nv_bfloat16* logits,
                                    int B, int V, int K, int num_sms, int* err, const LhPeer& peer,
                                    uint32_t* segk, int segk_stride, cudaStream_t stream) {
    CUtensorMap ma;
    if (!make_map(&ma, normed, B, K, kLhM)) return cudaErrorInvalidValue;
    switch (lm_head_tile(V, num_sms)) {
        case 176: return lm_head_go<176>(ma, W, logits, B, V, K, num_sms, err, peer, segk, segk_stride, stream);
        case 144: return lm_head_go<144>(ma, W, logits, B, V, K, num_sms, err, peer, segk, segk_stride, stream);
        case 128: return lm_head_go<128>(ma, W, logits, B, V, K, num_sms, err, peer, segk, segk_stride, stream);
        default: return lm_head_go<208>(ma, W, logits, B, V, K, num_sms, err, peer, segk, segk_stride, stream);
    }
}

// logits[B, V] = bf16(normed[B, K] . W[V, K]^T); B <= 128, K % 64 == 0.
// With segk, the epilogue also folds each row's raw maxima of the 256-column
// segments into segk[row * segk_stride + segment] (atomicMax of order keys;
// the buffer starts zeroed and the sampler's scan zeroes it again).
// Returns cudaErrorInvalidValue when a tensor map cannot be built.
cudaError_t launch_lm_head(const __nv_bfloat16* normed, const __nv_bfloat16* W, __nv_bfloat16* logits,
                           int B, int V, int K, int num_sms, int* err, cudaStream_t stream, uint32_t* segk,
                           int segk_stride) {
    LhPeer none;
    memset(&none, 0, sizeof(none));
    return lm_head_dispatch(normed, W, logits, B, V, K, num_sms, err, none, segk, segk_stride, stream);
}

// One vocabulary slice: logits of W_shard's `cols` rows for B <= 128 batch
// rows, each stored to the rank that samples it (see LhPeer).
cudaError_t launch_lm_head_shard(const __nv_bfloat16* normed, const __nv_bfloat16* W_shard, int B, int cols,
                                 int K, int num_sms, int* err, const LhPeer& peer, cudaStream_t stream) {
    return lm_head_dispatch(normed, W_shard, nullptr, B, cols, K, num_sms, err, peer, nullptr, 0, stream);
}

cudaError_t launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int B, int D,
                           cudaStream_t stream) {
    rmsnorm_rows_kernel<<<B, kNormThreads, 0, stream>>>(x, w, y, D, 1.0f / (float)D, 1e-6f);
    return cudaGetLastError();
}

}  // namespace qs
