// tc_gemm.cu — RaBitQ query preparation on the 5th-generation tensor cores.
//
// The two dense contractions of RaBitQ query preparation
// (RabitqQueryRotation::apply and ::centroid_distances,
// src/search/rabitq/rabitq_query_rotation.cuh:71-113, pedantic-FP32 cuBLAS
// SGEMMs in the reference) run here as one hand-written sm_100a GEMM:
//
//   C[m][n] = sum_k A[m][k] * B[n][k]        (both operands K-major, f32)
//
// * operands: TMA tiles (cp.async.bulk.tensor, 128-byte swizzle) of 128 rows
//   x 32 f32 (128 bytes) into a shared-memory ring of 192 KB, one mbarrier per
//   stage for "loaded" and one for "consumed";
// * math: one elected thread issues tcgen05.mma.cta_group::1.kind::tf32,
//   M = 128, N = 128 or 256, K = 8 per instruction, into 128 x N f32
//   accumulators in tensor memory; tcgen05.commit returns each stage to the
//   loader and hands each finished chunk to the promotion warps;
// * accumulation: chunks of 16 instructions go to one of two tensor-memory
//   buffers; eight promotion warps read each finished chunk with tcgen05.ld
//   (32x32b) into FP32 registers while the other buffer fills, then write
//   rows of C (plain, or the clamped centroid-distance form).
//
// FP32 accuracy ("3xTF32"): x = hi + lo with hi = tf32(x), lo = tf32(x - hi);
// A.B ~ lo_A.hi_B + hi_A.lo_B + hi_A.hi_B.  The three products are one GEMM
// over a K three times as long: A3 = [lo_A | hi_A | hi_A], B3 = [hi_B | lo_B |
// hi_B] (each segment padded to a multiple of 32 with zeros, the small
// corrections first), written to scratch by a split kernel.  One pass
// (plain TF32) skips the split.
//
// Every wait on an mbarrier is bounded; a wait that runs out sets the status
// word to GOFANN_ERR_TIMEOUT, skips the remaining work, waits (bounded) for
// the tensor-core operations it issued and frees its tensor memory.  No TMA
// multicast is used.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace gofann {
namespace {

constexpr int kBM = 128;            // tile rows (M of one MMA)
constexpr int kBK = 32;             // f32 elements per 128-byte swizzled row
constexpr int kTileA = kBM * kBK * 4;  // 16 KB
constexpr long long kSpinLimit = 1ll << 26;  // polls before a wait gives up

// Tile shape per variant: kBN columns (N of one MMA), a ring of stages that
// fits 192 KB, and kBN / 2 accumulator columns per promotion thread.
template <int kBN>
struct TileCfg {
    static constexpr int kTileB = kBN * kBK * 4;
    static constexpr int kStages = (192 * 1024) / (kTileA + kTileB);
    static constexpr int kHalfCols = kBN / 2;
    static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * (kTileA + kTileB) + 256;
    // Instruction descriptor (kind::tf32): D f32 (bits 4-5 = 1), A and B
    // tf32 (bits 7-9 and 10-12 = 2), both K-major, N >> 3 at bits 17-22,
    // M >> 4 at bits 24-28.
    static constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) |
                                       (static_cast<uint32_t>(kBN >> 3) << 17) |
                                       (static_cast<uint32_t>(kBM >> 4) << 24);
};

enum { kEpiPlain = 0, kEpiCentroidDist = 1 };

struct Epilogue {
    int mode;
    const float* row_norm;  // [M] (centroid distance)
    const float* col_norm;  // [N]
};

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// Bounded wait for the phase of `parity` to complete; false when it ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity)
{
    const uint32_t a = smem_u32(b);
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Shared-memory matrix descriptor of a K-major tile written by a 128-byte
// swizzled TMA copy: rows of 128 bytes, 8-row atoms 1024 bytes apart
// (stride byte offset), layout SWIZZLE_128B, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr)
{
    uint64_t d = static_cast<uint64_t>((saddr & 0x3ffffu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;            // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;    // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;            // version
    d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
    return d;
}
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's accumulator lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// One 128 x kBN tile of C per CTA.  Warps 0-7 promote and store (warp w
// reads accumulator lanes 32 (w % 4) .. + 31, columns kBN/2 (w / 4) ..),
// warp 8 lane 0 loads, warp 9 lane 0 issues the MMAs.
//
// The tensor core's accumulation into tensor memory drops low-order bits at
// each instruction, so a long K sum drifts (measured: 2.5e-4 relative after
// 1,536 instructions).  The MMAs therefore accumulate a chunk of K tiles
// at a time into one of two tensor-memory buffers, and the promotion warps
// add each finished chunk into FP32 registers while the MMAs fill the other
// buffer.  Chunks are kCoarseTiles K tiles (32 instructions) with plain
// additions before K tile `kahan_from`, and single K tiles (4 instructions)
// with compensated (Kahan) additions from there on, where the large products
// of a 3xTF32 GEMM come.
constexpr int kCoarseTiles = 8;  // K tiles per chunk before kahan_from (plain promotion)
constexpr int kGemmThreads = 320;

// kKahan: compensated promotion from K tile kahan_from on (the 128-column
// variant; the 256-column one keeps 128 accumulator registers per thread and
// promotes with plain additions only).
template <int kBN, bool kKahan>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int N,
                   int K, int kahan_from, float* __restrict__ C, long long ldc, Epilogue ep, int32_t* status)
{
    using Cfg = TileCfg<kBN>;
    constexpr int kStages = Cfg::kStages, kTileB = Cfg::kTileB, kHalfCols = Cfg::kHalfCols;
    constexpr uint32_t kTmemAlloc = 2 * kBN;  // two accumulator buffers
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* tiles_a = smem;
    unsigned char* tiles_b = smem + kStages * kTileA;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * (kTileA + kTileB));
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;   // [2] chunk of buffer b accumulated
    uint64_t* acc_empty = acc_full + 2;     // [2] buffer b promoted (8 warp arrivals)
    uint64_t* done = acc_empty + 2;         // every MMA issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int timed_out;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int kt_count = (K + kBK - 1) / kBK;
    const int fine_from = kahan_from < kt_count ? kahan_from : kt_count;
    const int coarse_chunks = (fine_from + kCoarseTiles - 1) / kCoarseTiles;
    const int chunks = coarse_chunks + (kt_count - fine_from);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        timed_out = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemAlloc)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 8) {
        if (lane == 0) {
            // loader: stage s is reused after the MMAs that read it committed
            for (int kt = 0; kt < kt_count; ++kt) {
                const int s = kt % kStages;
                if (kt >= kStages && !mbar_wait(&empty[s], ((kt / kStages) - 1) & 1)) {
                    atomicExch(&timed_out, 1);
                    break;
                }
                if (atomicAdd(&timed_out, 0)) break;
                mbar_expect_tx(&full[s], kTileA + kTileB);
                tma_load_2d(tiles_a + s * kTileA, &map_a, kt * kBK, m0, &full[s]);
                tma_load_2d(tiles_b + s * kTileB, &map_b, kt * kBK, n0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        if (lane == 0) {
            // MMA issuer: four K = 8 steps per 128-byte row, advancing the
            // start address 32 bytes inside the swizzle atom; chunk c into
            // buffer c % 2 once its previous chunk was promoted
            for (int kt = 0; kt < kt_count && !atomicAdd(&timed_out, 0); ++kt) {
                const int s = kt % kStages;
                const bool coarse = kt < fine_from;
                const int c = coarse ? kt / kCoarseTiles : coarse_chunks + (kt - fine_from), b = c & 1;
                const bool first = coarse ? kt % kCoarseTiles == 0 : true;
                const bool last = kt == kt_count - 1 ||
                                  (coarse ? (kt % kCoarseTiles == kCoarseTiles - 1 || kt + 1 == fine_from) : true);
                if (first && c >= 2 && !mbar_wait(&acc_empty[b], ((c >> 1) - 1) & 1)) {
                    atomicExch(&timed_out, 1);
                    break;
                }
                if (!mbar_wait(&full[s], (kt / kStages) & 1)) {
                    atomicExch(&timed_out, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(tiles_a + s * kTileA), b0 = smem_u32(tiles_b + s * kTileB);
                const uint32_t d = tmem + static_cast<uint32_t>(b * kBN);
#pragma unroll
                for (int k = 0; k < kBK / 8; ++k)
                    umma_tf32(d, umma_desc(a0 + 32 * k), umma_desc(b0 + 32 * k), Cfg::kIdesc, (!first || k != 0) ? 1u : 0u);
                umma_commit(&empty[s]);
                if (last) umma_commit(&acc_full[b]);
            }
            umma_commit(done);  // arrives once every MMA issued above has completed
        }
        __syncwarp();
    } else {
        // promotion: kHalfCols columns of one accumulator lane per thread
        const int quarter = warp & 3, half = warp >> 2;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        float acc[kHalfCols], comp[kKahan ? kHalfCols : 1];
#pragma unroll
        for (int i = 0; i < kHalfCols; ++i) acc[i] = 0.0f;
#pragma unroll
        for (int i = 0; i < (kKahan ? kHalfCols : 1); ++i) comp[i] = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            const int b = c & 1;
            if (!mbar_wait(&acc_full[b], (c >> 1) & 1)) {
                atomicExch(&timed_out, 1);
                break;
            }
            tc_fence_after();
            const bool kahan = kKahan && c >= coarse_chunks;
#pragma unroll
            for (int j = 0; j < kHalfCols / 32; ++j) {
                float v[32];
                tmem_ld32(tmem + lane_base + static_cast<uint32_t>(b * kBN + half * kHalfCols + j * 32), v);
                if (kahan) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        float& cp = comp[kKahan ? j * 32 + i : 0];
                        const float y = __fsub_rn(v[i], cp);
                        const float t = __fadd_rn(acc[j * 32 + i], y);
                        cp = __fsub_rn(__fsub_rn(t, acc[j * 32 + i]), y);
                        acc[j * 32 + i] = t;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[j * 32 + i] = __fadd_rn(acc[j * 32 + i], v[i]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        const int row = m0 + quarter * 32 + lane;
        if (!atomicAdd(&timed_out, 0) && row < M) {
            const float rn = ep.mode == kEpiCentroidDist ? ep.row_norm[row] : 0.0f;
            float* dst = C + static_cast<long long>(row) * ldc + n0 + half * kHalfCols;
#pragma unroll
            for (int i = 0; i < kHalfCols; ++i) {
                const int col = n0 + half * kHalfCols + i;
                if (col < N) {
                    float x = acc[i];
                    if (ep.mode == kEpiCentroidDist)
                        x = fmaxf(0.0f, __fadd_rn(__fadd_rn(__fmul_rn(-2.0f, x), rn), ep.col_norm[col]));
                    dst[i] = x;
                }
            }
        }
    }

    // every issued MMA must have completed before the tensor memory is freed
    if (!mbar_wait(done, 0)) atomicExch(&timed_out, 1);
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && timed_out && status) atomicExch(status, GOFANN_ERR_TIMEOUT);
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemAlloc) : "memory");
}

// tf32 rounding (round to nearest, ties away from zero): an f32 whose low 13
// mantissa bits are zero, exactly what the tensor core reads.
__device__ __forceinline__ float to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Writes the operand of a 3xTF32 GEMM: row r of dst (3 * kp columns) holds
// three segments of kp values from row r of the source; `order` 0 = (lo,
// hi, hi) for A, 1 = (hi, lo, hi) for B.  The source element of (r, k) is
// src[r * ld + k] (row_major) or src[k * ld + r] (transposed); k >= K and
// r >= rows read as zero.  32 x 32 tiles through shared memory keep both
// sides coalesced.
__global__ void split3_kernel(const float* __restrict__ src, int rows, int K, long long ld, bool transposed, int kp,
                              int order, float* __restrict__ dst)
{
    __shared__ float tile[32][33];
    const int r0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    for (int i = ty; i < 32; i += 8) {
        float x = 0.0f;
        if (transposed) {
            const int k = k0 + i, r = r0 + tx;
            if (k < K && r < rows) x = src[static_cast<long long>(k) * ld + r];
            tile[tx][i] = x;
        } else {
            const int r = r0 + i, k = k0 + tx;
            if (k < K && r < rows) x = src[static_cast<long long>(r) * ld + k];
            tile[i][tx] = x;
        }
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, k = k0 + tx;
        if (r >= rows || k >= kp) continue;
        const float x = tile[i][tx];
        const float hi = to_tf32(x);
        const float lo = to_tf32(__fsub_rn(x, hi));
        float* d = dst + static_cast<long long>(r) * 3 * kp;
        d[k] = order == 0 ? lo : hi;
        d[kp + k] = order == 0 ? hi : lo;
        d[2 * kp + k] = hi;
    }
}

// Copy of a row-major operand (or the transpose of one) into a K-major
// buffer padded to kp columns, for the one-pass path.
__global__ void pack_kernel(const float* __restrict__ src, int rows, int K, long long ld, bool transposed, int kp,
                            float* __restrict__ dst)
{
    __shared__ float tile[32][33];
    const int r0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        float x = 0.0f;
        if (transposed) {
            const int k = k0 + i, r = r0 + tx;
            if (k < K && r < rows) x = src[static_cast<long long>(k) * ld + r];
            tile[tx][i] = x;
        } else {
            const int r = r0 + i, k = k0 + tx;
            if (k < K && r < rows) x = src[static_cast<long long>(r) * ld + k];
            tile[i][tx] = x;
        }
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, k = k0 + tx;
        if (r < rows && k < kp) dst[static_cast<long long>(r) * kp + k] = tile[i][tx];
    }
}

// Squared norms of rows (sequential fma per thread over a strided part, then
// a shared-memory tree; FP32).
__global__ void __launch_bounds__(256) row_norms_kernel(const float* __restrict__ x, int rows, int dim,
                                                        float* __restrict__ out)
{
    __shared__ float part[256];
    const int r = blockIdx.x;
    float s = 0.0f;
    for (int d = threadIdx.x; d < dim; d += 256) {
        const float v = x[static_cast<long long>(r) * dim + d];
        s = __fmaf_rn(v, v, s);
    }
    part[threadIdx.x] = s;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) part[threadIdx.x] = __fadd_rn(part[threadIdx.x], part[threadIdx.x + stride]);
        __syncthreads();
    }
    if (threadIdx.x == 0) out[r] = part[0];
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
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

// Tensor map of a row-major f32 matrix [rows][cols] (cols a multiple of 4,
// base 16-byte aligned) read in boxes of box_rows x 32 with 128-byte swizzle.
int make_map(CUtensorMap* map, const float* base, long long rows, long long cols, int box_rows)
{
    auto fn = encode_fn();
    if (!fn) return fail(GOFANN_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GOFANN_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return GOFANN_OK;
}

// C[M][N] = A[M][K] . B[N][K]^T over K-major f32 buffers (K a multiple of
// 32); compensated promotion from K tile kahan_from on in the kKahan variant.
template <int kBN, bool kKahan>
int launch_gemm(const float* a, const float* b, int M, int N, int K, int kahan_from, float* c, long long ldc,
                Epilogue ep, int32_t* status, cudaStream_t s)
{
    CUtensorMap ma, mb;
    int st = make_map(&ma, a, M, K, kBM);
    if (st != GOFANN_OK) return st;
    st = make_map(&mb, b, N, K, kBN);
    if (st != GOFANN_OK) return st;
    const size_t smem = TileCfg<kBN>::kSmem;
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<kBN, kKahan>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "tc_gemm: shared memory attribute");
    const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
    tc_gemm_kernel<kBN, kKahan><<<grid, kGemmThreads, smem, s>>>(ma, mb, M, N, K, kahan_from, c, ldc, ep, status);
    GOFANN_CHECK_LAUNCH("tc_gemm_kernel");
    return GOFANN_OK;
}

inline long long round32(long long x) { return (x + 31) / 32 * 32; }
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Scratch layout of one preparation GEMM: the two prepared operands, then
// two norm vectors.
struct PrepScratch {
    size_t a_bytes, b_bytes, norm_bytes, total;
};
PrepScratch prep_scratch(uint32_t rows, uint32_t k, uint32_t cols, int precision)
{
    const long long kp = round32(k);
    const long long kk = precision == GOFANN_GEMM_TF32X3 ? 3 * kp : kp;
    PrepScratch p;
    p.a_bytes = align256(static_cast<size_t>(rows) * kk * 4);
    p.b_bytes = align256(static_cast<size_t>(cols) * kk * 4);
    p.norm_bytes = align256(static_cast<size_t>(rows + cols) * 4);
    p.total = p.a_bytes + p.b_bytes + p.norm_bytes;
    return p;
}

// Prepares A (rows x k, row-major, leading dim lda) and B (cols x k; from a
// row-major [cols][k] buffer, or transposed from [k][cols]) in scratch and
// runs the GEMM.
int prep_gemm(const float* a, uint32_t rows, long long lda, const float* b, bool b_transposed, long long ldb,
              uint32_t cols, uint32_t k, int precision, float* c, long long ldc, Epilogue ep, void* scratch,
              int32_t* status, cudaStream_t s)
{
    const PrepScratch ps = prep_scratch(rows, k, cols, precision);
    unsigned char* base = static_cast<unsigned char*>(scratch);
    float* a2 = reinterpret_cast<float*>(base);
    float* b2 = reinterpret_cast<float*>(base + ps.a_bytes);
    const int kp = static_cast<int>(round32(k));
    const dim3 blk(256);
    const dim3 ga((kp + 31) / 32, (rows + 31) / 32), gb((kp + 31) / 32, (cols + 31) / 32);
    if (precision == GOFANN_GEMM_TF32X3) {
        split3_kernel<<<ga, blk, 0, s>>>(a, static_cast<int>(rows), static_cast<int>(k), lda, false, kp, 0, a2);
        split3_kernel<<<gb, blk, 0, s>>>(b, static_cast<int>(cols), static_cast<int>(k), ldb, b_transposed, kp, 1, b2);
    } else {
        pack_kernel<<<ga, blk, 0, s>>>(a, static_cast<int>(rows), static_cast<int>(k), lda, false, kp, a2);
        pack_kernel<<<gb, blk, 0, s>>>(b, static_cast<int>(cols), static_cast<int>(k), ldb, b_transposed, kp, b2);
    }
    GOFANN_CHECK_LAUNCH("tc_gemm operand preparation");
    const int kk = precision == GOFANN_GEMM_TF32X3 ? 3 * kp : kp;
    // 3xTF32: 128-column tiles, the hi.hi segment (the last third) promoted
    // with compensation; one pass: 256-column tiles, plain promotion
    if (precision == GOFANN_GEMM_TF32X3)
        return launch_gemm<128, true>(a2, b2, static_cast<int>(rows), static_cast<int>(cols), kk, 2 * kp / kBK, c,
                                      ldc, ep, status, s);
    return launch_gemm<256, false>(a2, b2, static_cast<int>(rows), static_cast<int>(cols), kk, kk / kBK, c, ldc, ep,
                                   status, s);
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

size_t gofann_rabitq_gemm_scratch_bytes(uint32_t rows, uint32_t k, uint32_t cols, int precision)
{
    return prep_scratch(rows, k, cols, precision).total;
}

int gofann_rabitq_rotate(const float* queries, uint32_t n, uint32_t dim, const float* rotation, uint32_t padded_dim,
                         int precision, float* rotated_out, void* scratch, size_t scratch_bytes, int32_t* status,
                         void* stream)
{
    if (!queries || !rotation || !rotated_out || !scratch) return fail(GOFANN_ERR_INVALID, "rabitq_rotate: null pointer");
    if (precision != GOFANN_GEMM_TF32 && precision != GOFANN_GEMM_TF32X3)
        return fail(GOFANN_ERR_INVALID, "rabitq_rotate: unknown precision %d", precision);
    if (dim == 0 || padded_dim < dim)
        return fail(GOFANN_ERR_INVALID, "rabitq_rotate: dim %u / padded_dim %u (padded_dim must be >= dim > 0)", dim,
                    padded_dim);
    if (n == 0) return GOFANN_OK;
    if ((reinterpret_cast<uintptr_t>(scratch) & 255) != 0)
        return fail(GOFANN_ERR_INVALID, "rabitq_rotate: scratch must be 256-byte aligned");
    const size_t need = prep_scratch(n, dim, padded_dim, precision).total;
    if (scratch_bytes < need)
        return fail(GOFANN_ERR_CAPACITY, "rabitq_rotate: scratch of %zu bytes, %zu needed", scratch_bytes, need);
    // q' = q . R: A = queries [n][dim], B[p][d] = R[d][p] (the transpose of
    // the [dim][padded_dim] rotation)
    Epilogue ep{kEpiPlain, nullptr, nullptr};
    return prep_gemm(queries, n, dim, rotation, true, padded_dim, padded_dim, dim, precision, rotated_out, padded_dim,
                     ep, scratch, status, as_stream(stream));
}

int gofann_rabitq_centroid_dist_tc(const float* rotated, uint32_t n, const float* anchors, uint32_t num_anchors,
                                   uint32_t padded_dim, int precision, float* gdist_out, void* scratch,
                                   size_t scratch_bytes, int32_t* status, void* stream)
{
    if (!rotated || !anchors || !gdist_out || !scratch)
        return fail(GOFANN_ERR_INVALID, "rabitq_centroid_dist_tc: null pointer");
    if (precision != GOFANN_GEMM_TF32 && precision != GOFANN_GEMM_TF32X3)
        return fail(GOFANN_ERR_INVALID, "rabitq_centroid_dist_tc: unknown precision %d", precision);
    if (padded_dim == 0) return fail(GOFANN_ERR_INVALID, "rabitq_centroid_dist_tc: padded_dim is zero");
    if (n == 0 || num_anchors == 0) return GOFANN_OK;
    if ((reinterpret_cast<uintptr_t>(scratch) & 255) != 0)
        return fail(GOFANN_ERR_INVALID, "rabitq_centroid_dist_tc: scratch must be 256-byte aligned");
    const PrepScratch ps = prep_scratch(n, padded_dim, num_anchors, precision);
    if (scratch_bytes < ps.total)
        return fail(GOFANN_ERR_CAPACITY, "rabitq_centroid_dist_tc: scratch of %zu bytes, %zu needed", scratch_bytes,
                    ps.total);
    float* norms = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + ps.a_bytes + ps.b_bytes);
    cudaStream_t s = as_stream(stream);
    row_norms_kernel<<<n, 256, 0, s>>>(rotated, static_cast<int>(n), static_cast<int>(padded_dim), norms);
    row_norms_kernel<<<num_anchors, 256, 0, s>>>(anchors, static_cast<int>(num_anchors), static_cast<int>(padded_dim),
                                                 norms + n);
    GOFANN_CHECK_LAUNCH("row_norms_kernel");
    // gdist[q][a] = max(0, -2 q.c + |q|^2 + |c|^2): A = rotated queries, B = anchors (both [.][padded_dim])
    Epilogue ep{kEpiCentroidDist, norms, norms + n};
    return prep_gemm(rotated, n, padded_dim, anchors, false, padded_dim, num_anchors, padded_dim, precision, gdist_out,
                     num_anchors, ep, scratch, status, s);
}

}  // extern "C"
