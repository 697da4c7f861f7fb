// The pruned 2D real forward (rfft2_truncated) of 128 x 128 fields with its row stage as a GEMM
// on the 5th-generation tensor cores (tcgen05), in FP32 accuracy through split TF32.
//
// Pruning makes the row stage a skinny matrix product: of each real row's 65 outputs only the
// first m2 <= 16 are kept, and
//   R[n1, k] = sum_n2 x[n1, n2] exp(-2 pi i k n2 / 128),   k < m2,
// is, for one field, D = X F^T with X the 128 x 128 field (M = 128 rows, K = 128) and F the
// 32 x 128 real matrix of cos and -sin rows (N = 32). The FFT engine computes all 64 packed
// outputs of a row and discards most of them; the GEMM computes only the kept ones, and the
// field's data never passes through shared-memory exchanges.
//
// Precision: tcgen05 kind::tf32 multiplies TF32 values (10 fraction bits). Both operands are
// split into a hi part (the value rounded to TF32) and a lo part (the remainder, rounded to
// TF32), and three products are kept: x_hi F_hi, x_hi F_lo and x_lo F_hi; the dropped x_lo F_lo
// is 2^-22 of the product. F's parts are built once on the host in double precision
// (twiddles::tf32_dft_rows: rows cos hi, -sin hi, cos lo, -sin lo). Per chunk of 8 values of K,
// one MMA with N = 64 (all four F row blocks) gives x_hi F_hi in accumulator columns 0-31 and
// x_hi F_lo in 32-63, and one with N = 32 gives x_lo F_hi in 64-95: the large products have an
// accumulator of their own, so the small ones are not rounded at its magnitude, and the three are
// added in FP32 registers at the end.
//
// The column stage (128-point transforms of the m2 kept columns, only the 2 m1 kept rows
// written) is the radix-8 engine's, as in the FP32 pruned kernel (pruned2d.cuh).
//
// Data flow, per CTA (one per SM, persistent over fields), warp-specialized:
//   - warp 0: TMA loads of the field's rows in chunks of 32 values (boxes of 128 rows x 128 bytes,
//     128-byte swizzle), 10 chunks (160 KiB) in flight: a load takes about 2.5 us from issue to
//     arrival at this kernel's bandwidth, and the stages in flight set the bandwidth;
//   - warps 2-9, two sets of 4 taking alternate chunks: each thread owns one row (TMEM lane): it
//     reads its 32 values of a chunk from shared memory (then releases the stage), splits them,
//     and stores the hi and lo parts into the chunk's A operand in tensor memory (tcgen05.st;
//     TMEM lanes are rows, columns are K), 4 chunk stages;
//   - warp 1: one elected lane issues the MMAs (A from tensor memory, F from shared memory) into
//     one of two field accumulators and commits them;
//   - warps 10-13 and 14-17: two column groups taking alternate fields. A group reads its field's
//     accumulators (one row per thread), adds the three products, writes the 128 x 16 complex
//     tile to shared memory, runs the column passes (named barriers over its 128 threads) and
//     stores the kept modes.
// Roles meet only on mbarriers. Every wait is bounded and its outcome made uniform over the
// threads that act on it; a wait that gives up records a fault code, the CTA waits (bounded) for
// the copies and MMAs it issued, frees its tensor memory and returns. The tensor map covers this
// GPU's own input, and no load is multicast.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "launch.cuh"
#include "pruned2d.cuh"
#include "tma.cuh"
#include "twiddles.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cstdint>
#include <mutex>

namespace spectral {
namespace {

constexpr int kN1 = 128;                           // rows per field: the MMA's M, one TMEM lane each
constexpr int kN2 = 128;                           // values per row: the GEMM's K
constexpr int kMaxM2 = twiddles::kTf32DftOutputs;  // 16 kept outputs per row at most
constexpr int kKc = 32;                            // values per chunk: 128 bytes, one swizzle span
constexpr int kChunks = kN2 / kKc;
constexpr int kSteps = kKc / 8;                    // MMAs of K = 8 per chunk and product
constexpr int kFRows = 4 * kMaxM2;                 // cos hi, -sin hi, cos lo, -sin lo
constexpr int kLbo = kFRows / 8 * 128;             // F: bytes between core matrices along K
constexpr int kSbo = 128;                          // F: bytes between 8-row groups
constexpr int kFBytes = kN2 / 4 * kLbo;            // 32 KiB
constexpr int kStages = 10;                        // x chunks in shared memory (160 KiB in flight)
constexpr int kAStages = 4;                        // split chunks in tensor memory
constexpr int kBoxBytes = kN1 * kKc * 4;           // 16 KiB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDCols = 128;                   // a field's accumulator: 64 + 32 columns used
constexpr uint32_t kACol0 = 2 * kDCols;            // the split chunk stages follow the two fields
constexpr uint32_t kACols = 2 * kKc;               // hi 32 + lo 32 columns
static_assert(kACol0 + kAStages * kACols <= kTmemCols, "tensor memory");

using CP = engine::PlanFor<kN1>;                   // 128-point columns: E = 16 values per thread
constexpr int kCW = kN1 / CP::P;                   // columns in flight per group of 128 threads
static_assert(kCW == kMaxM2, "one column group covers every kept column");
constexpr int kColEntries = kN1 * kCW;             // a group's [row][column] tile (float2)
constexpr int kTwEntries = (CP::TW + 1) & ~1;

constexpr int kSplitWarp0 = 2;                     // two sets of 4 split warps (one per TMEM lane
constexpr int kSplitSets = 2;                      // quarter) taking alternate chunks: warps 2-9
constexpr int kColWarp0 = kSplitWarp0 + 4 * kSplitSets;
constexpr int kGroups = 2;
constexpr int kThreads = (kColWarp0 + 4 * kGroups) * 32;  // 576

constexpr int kOffX = 0;
constexpr int kOffF = kOffX + kStages * kBoxBytes;
constexpr int kOffCol = kOffF + kFBytes;
constexpr int kOffTw = kOffCol + kGroups * kColEntries * 8;
constexpr int kOffBar = kOffTw + kTwEntries * 8;
constexpr int kBars = 2 * kStages + 2 * kAStages + 2 * kGroups;
constexpr int kSmemBytes = kOffBar + kBars * 8 + 16 + 1024;  // + slack for the 1 KiB aligned base
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kSmemBytes > 114 * 1024, "one CTA per SM: the CTA takes all of tensor memory");

// tcgen05.mma kind::tf32 instruction descriptor: F32 accumulator, TF32 A and B, both K-major,
// M = 128, N = n (bits: c_format 4-5, a_format 7-9, b_format 10-12, N / 8 at 17-22, M / 16 at 24-28).
constexpr uint32_t idesc(int n)
{
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n / 8) << 17)
           | (static_cast<uint32_t>(kN1 / 16) << 24);
}

// Shared-memory matrix descriptor of F at `addr`: leading (K) and stride (rows) byte offsets in
// 16-byte units, version 1 at bit 46, no swizzle.
__device__ __forceinline__ uint64_t f_desc(uint32_t addr)
{
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((kLbo >> 4) & 0x3FFF) << 16)
           | (static_cast<uint64_t>((kSbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

template <int Lbo>
__device__ __forceinline__ uint64_t f_desc_lbo(uint32_t addr)
{
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((Lbo >> 4) & 0x3FFF) << 16)
           | (static_cast<uint64_t>((kSbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ float tf32_round(float a)
{
    return __uint_as_float((__float_as_uint(a) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tma::smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(tma::smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(tma::smem_addr(bar))
        : "memory");
}

// D (+)= A B^T with A (128 x 8 TF32) in tensor memory at column `a` and B (N x 8) in shared
// memory.
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t desc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(desc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     tma::smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes, one lane per thread (no wait).
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Waits for this thread's tensor-memory loads. The registers a load wrote are in-out operands of
// the wait, so the compiler places every use of them after it.
__device__ __forceinline__ void tmem_wait_load(uint32_t (&r)[32])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// Stores 32 consecutive 32-bit columns of this warp's 32 TMEM lanes, one lane per thread.
__device__ __forceinline__ void tmem_store32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_store() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// True in every thread of the column group on named barrier Id when `ok` holds in all of its 128
// threads (a barrier with an AND reduction: the group then takes the same branch).
template <int Id>
__device__ __forceinline__ bool group_all(bool ok)
{
    uint32_t r = 0;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(ok)), "n"(Id)
        : "memory");
    return r != 0;
}

// One column group's share: the fields i = G, G + kGroups, .. of this CTA, in accumulator G.
template <int G>
__device__ __forceinline__ bool column_group(uint64_t* dfull, uint64_t* dempty, uint32_t tmem, float2* tile,
                                             const float2* twc, float2* __restrict__ modes, long long nf,
                                             int m1, int m2)
{
    constexpr int kSync = ((1 + G) << 10) | 128;  // named barrier 1 + G over the group's 128 threads
    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int gt = tid - (kColWarp0 + 4 * G) * 32;  // 0 .. 127
    const int r = (warp & 3) * 32 + lane;           // this thread's row (TMEM lane)
    const int cc = gt % kCW;
    const int ct = gt / kCW;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    for (long long i = G; i < nf; i += kGroups) {
        const bool ok = tma::mbar_wait(&dfull[G], static_cast<unsigned>(i / kGroups) & 1u);
        if (!group_all<(kSync >> 10)>(ok)) {
            return false;
        }
        fence_after_sync();
        uint32_t a[32], b[32];
        const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(G) * kDCols;
        tmem_load32(acc + 32, a);    // x_hi cos_lo (0-15), x_hi (-sin)_lo (16-31)
        tmem_load32(acc + 64, b);    // x_lo cos_hi, x_lo (-sin)_hi
        tmem_wait_load(a);
        tmem_wait_load(b);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            a[k] = __float_as_uint(__uint_as_float(a[k]) + __uint_as_float(b[k]));
        }
        tmem_load32(acc, b);         // x_hi cos_hi, x_hi (-sin)_hi
        tmem_wait_load(b);
        fence_before_sync();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&dempty[G]);  // the accumulator may take the group's next field
        }
        // Row r's 16 outputs into the tile, column k at k ^ (r mod 16): a warp's 32 rows then
        // fall on 16 distinct bank pairs for each k, and a row stays one 128-byte line.
#pragma unroll
        for (int k = 0; k < kCW; ++k) {
            const float re = __uint_as_float(b[k]) + __uint_as_float(a[k]);
            const float im = __uint_as_float(b[kCW + k]) + __uint_as_float(a[kCW + k]);
            tile[r * kCW + (k ^ (r & 15))] = make_float2(re, im);
        }
        engine::exchange_sync<1, kSync>();
        float2 v[CP::E];
#pragma unroll
        for (int e = 0; e < CP::E; ++e) {
            const int row = ct + e * CP::P;
            v[e] = tile[row * kCW + (cc ^ (row & 15))];
        }
        engine::exchange_sync<1, kSync>();
        engine::run_passes<CP, false, 8, kCW, kSync>(v, ct, tile + cc, twc);
        if (cc < m2) {
            const long long f = static_cast<long long>(blockIdx.x) + i * gridDim.x;
            float2* mf = modes + f * (2LL * m1 * m2);
#pragma unroll
            for (int e = 0; e < CP::E; ++e) {
                const int row = engine::mode_row(ct + e * CP::P, kN1, m1);
                if (row >= 0) {
                    mf[row * m2 + cc] = v[e];
                }
            }
        }
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    pruned_tc_forward_kernel(const __grid_constant__ CUtensorMap map_x, float2* __restrict__ modes,
                             long long fields, int m1, int m2, const float2* __restrict__ f_rows,
                             const float2* __restrict__ twc_g, unsigned* fault)
{
    allow_next_grid();
    extern __shared__ unsigned char smem_base[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_base) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* xs = smem + kOffX;
    unsigned char* fs = smem + kOffF;
    auto* colbuf = reinterpret_cast<float2*>(smem + kOffCol);
    auto* twc = reinterpret_cast<float2*>(smem + kOffTw);
    auto* sfull = reinterpret_cast<uint64_t*>(smem + kOffBar);  // chunk landed (TMA)
    uint64_t* sempty = sfull + kStages;                          // chunk read by the 4 split warps
    uint64_t* afull = sempty + kStages;                          // split chunk stored (4 warps)
    uint64_t* aempty = afull + kAStages;                         // its MMAs completed
    uint64_t* dfull = aempty + kAStages;                         // a field's MMAs completed
    uint64_t* dempty = dfull + kGroups;                          // its accumulator read (4 warps)
    auto* tmem_slot = reinterpret_cast<uint32_t*>(dempty + kGroups);

    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int lane = tid & 31;

    // F in shared memory (the tensor core reads it through the async proxy) and the column
    // twiddles, once per CTA.
    for (int i = tid; i < kFBytes / 8; i += kThreads) {
        reinterpret_cast<float2*>(fs)[i] = f_rows[i];
    }
    engine::fill_pass_twiddles<CP, true>(twc, twc_g);
    tma::fence_proxy_async();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tma::smem_addr(tmem_slot)),
                     "n"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            tma::mbar_init(&sfull[s], 1);
            tma::mbar_init(&sempty[s], 4);
        }
        for (int a = 0; a < kAStages; ++a) {
            tma::mbar_init(&afull[a], 4);
            tma::mbar_init(&aempty[a], 1);
        }
        for (int d = 0; d < kGroups; ++d) {
            tma::mbar_init(&dfull[d], 1);
            tma::mbar_init(&dempty[d], 4);
        }
        tma::fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // The set-up above reads only host-built tables and this CTA's own resources, so it overlaps
    // the previous kernel's tail; from here on global data another kernel may write is touched.
    wait_for_previous_grid();

    const long long bx = blockIdx.x;
    const long long nf = fields > bx ? (fields - 1 - bx) / gridDim.x + 1 : 0;  // this CTA's fields
    const long long chunks = nf * kChunks;
    bool failed = false;
    long long issued = 0;     // warp 0: chunks whose TMA load was issued
    long long committed = 0;  // warp 1: chunks whose MMAs were committed

    if (warp == 0) {
        for (long long q = 0; q < chunks; ++q) {
            const int s = static_cast<int>(q % kStages);
            const bool ok = q < kStages || tma::mbar_wait(&sempty[s], static_cast<unsigned>(q / kStages - 1) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                failed = true;
                break;
            }
            const long long f = bx + (q / kChunks) * gridDim.x;
            const int c = static_cast<int>(q % kChunks);
            if (elect_one()) {
                tma::mbar_arrive_expect_tx(&sfull[s], kBoxBytes);
                tma_load_2d(xs + s * kBoxBytes, &map_x, c * kKc, static_cast<int>(f * kN1), &sfull[s]);
            }
            __syncwarp();
            ++issued;
        }
    } else if (warp == 1) {
        const uint32_t f0 = tma::smem_addr(fs);
        for (long long i = 0; i < nf && !failed; ++i) {
            const uint32_t d = static_cast<uint32_t>(i % kGroups);
            bool ok = i < kGroups || tma::mbar_wait(&dempty[d], static_cast<unsigned>(i / kGroups - 1) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                failed = true;
                break;
            }
            for (int c = 0; c < kChunks; ++c) {
                const long long q = i * kChunks + c;
                const int a = static_cast<int>(q % kAStages);
                ok = tma::mbar_wait(&afull[a], static_cast<unsigned>(q / kAStages) & 1u);
                if (!__all_sync(0xffffffffu, ok)) {
                    failed = true;
                    break;
                }
                fence_after_sync();
                if (elect_one()) {
                    const uint32_t dcol = tmem + d * kDCols;
                    const uint32_t acol = tmem + kACol0 + static_cast<uint32_t>(a) * kACols;
#pragma unroll
                    for (int jj = 0; jj < kSteps; ++jj) {
                        const uint64_t b = f_desc(f0 + static_cast<uint32_t>((c * kSteps + jj) * 2 * kLbo));
                        const uint32_t acc = (c | jj) != 0 ? 1u : 0u;
                        mma_ts(dcol, acol + 8 * jj, b, idesc(4 * kMaxM2), acc);            // x_hi [F_hi; F_lo]
                        mma_ts(dcol + 64, acol + kKc + 8 * jj, b, idesc(2 * kMaxM2), acc);  // x_lo F_hi
                    }
                    mma_commit(&aempty[a]);
                    if (c == kChunks - 1) {
                        mma_commit(&dfull[d]);
                    }
                }
                __syncwarp();
                ++committed;
            }
        }
    } else if (warp < kColWarp0) {
        // Split warps: thread = row r of the field = TMEM lane r; set `set` takes the chunks
        // q = set, set + kSplitSets, ..
        const int r = (warp & 3) * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const int set = (warp - kSplitWarp0) / 4;
        for (long long q = set; q < chunks; q += kSplitSets) {
            const int s = static_cast<int>(q % kStages);
            const int a = static_cast<int>(q % kAStages);
            bool ok = tma::mbar_wait(&sfull[s], static_cast<unsigned>(q / kStages) & 1u);
            if (ok && q >= kAStages) {
                ok = tma::mbar_wait(&aempty[a], static_cast<unsigned>(q / kAStages - 1) & 1u);
            }
            if (!__all_sync(0xffffffffu, ok)) {
                failed = true;
                break;
            }
            fence_after_sync();
            // Row r of the box: 128 bytes at r * 128, 16-byte piece j stored at piece j ^ (r mod 8)
            // (the TMA's 128-byte swizzle): a quarter-warp's 8 rows read 8 distinct bank groups.
            const unsigned char* row = xs + s * kBoxBytes + r * 128;
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v = *reinterpret_cast<const float4*>(row + ((j ^ (r & 7)) << 4));
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float h = tf32_round(e[t]);
                    hi[4 * j + t] = __float_as_uint(h);
                    lo[4 * j + t] = __float_as_uint(tf32_round(e[t] - h));
                }
            }
            // The chunk's values are in registers: its stage may take the next load already.
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sempty[s]);
            }
            const uint32_t acol = tmem + lane_base + kACol0 + static_cast<uint32_t>(a) * kACols;
            tmem_store32(acol, hi);
            tmem_store32(acol + kKc, lo);
            tmem_wait_store();
            fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&afull[a]);
            }
        }
    } else if (warp < kColWarp0 + 4) {
        failed = !column_group<0>(dfull, dempty, tmem, colbuf, twc, modes, nf, m1, m2);
    } else {
        failed = !column_group<1>(dfull, dempty, tmem, colbuf + kColEntries, twc, modes, nf, m1, m2);
    }

    if (__syncthreads_or(failed)) {
        // Let what this CTA issued finish (bounded) before its shared and tensor memory go: the
        // last kStages loads, and the last MMA commit (it tracks every earlier MMA).
        bool drained = true;
        if (tid == 0) {
            atomicOr(fault, tma::kFaultWaitTimeout);
            for (long long q = issued > kStages ? issued - kStages : 0; q < issued; ++q) {
                drained = tma::mbar_wait(&sfull[q % kStages], static_cast<unsigned>(q / kStages) & 1u) && drained;
            }
        }
        if (tid == 32 && committed > 0) {
            const long long q = committed - 1;
            drained = tma::mbar_wait(&aempty[q % kAStages], static_cast<unsigned>(q / kAStages) & 1u) && drained;
        }
        if (!drained) {
            atomicOr(fault, tma::kFaultDrainTimeout);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols) : "memory");
    }
}

// --- the inverse (irfft2_from_modes) ------------------------------------------------------------
//
// Columns first: the m2 kept columns' 128-point inverse transforms (the radix-8 engine, from the
// 2 m1 kept rows), which leave R[n1, k] for every row n1 and k < m2. Then each row's real inverse
//   y[n1, n2] = sum_k c_k (Re R[n1, k] cos(2 pi k n2 / 128) - Im R[n1, k] sin(2 pi k n2 / 128)) / 128^2,
// c_0 = 1 and c_k = 2 otherwise (the Hermitian partner of each kept column; Im R[n1, 0] meets
// sin 0 = 0 and drops out as a real inverse drops it), is Y = A' C'^T: A' (M = 128 rows, K = 32)
// holds c_k Re R / 128^2 and -c_k Im R / 128^2 (exact scalings by powers of two), C' (N = 128
// output positions, K = 32) holds cos and sin (twiddles::tf32_idft_rows). Both are split into
// TF32 hi and lo parts; the three products x_hi C_hi, x_hi C_lo and x_lo C_hi accumulate in one
// accumulator (32 terms per output: its per-MMA rounding stays at the FP32 level).
//
// Warps: 0 issues the MMAs (3 per 8 values of K, N = 128); 1-4 (the epilogue) read a field's
// accumulator (one output row per thread, 32 columns at a time), stage the rows in shared memory
// in the 128-byte swizzled box layout and store each 128 x 32 box with one TMA store; 5-8 and
// 9-12, two column groups on alternate fields, load the kept modes (the next field's a field
// ahead), run the column passes, turn the column-major result into rows through a shared-memory
// tile and store each row's split A' into tensor memory. Accumulators: 2 x 128 columns; A': 4
// fields x 64 columns.

constexpr int kIK = 2 * kMaxM2;                    // 32: cos and sin coefficients of a row
constexpr int kIFRows = 2 * kN2;                   // C' hi rows, then lo rows
constexpr int kILbo = kIFRows / 8 * 128;           // 4 KiB
constexpr int kIFBytes = kIK / 4 * kILbo;          // 32 KiB
constexpr int kIDStages = 2;
constexpr int kIAStages = 4;
constexpr uint32_t kIDCols = 128;
constexpr uint32_t kIACol0 = kIDStages * kIDCols;
constexpr uint32_t kIACols = 2 * kIK;              // hi 32 + lo 32
static_assert(kIACol0 + kIAStages * kIACols <= kTmemCols, "tensor memory");
constexpr int kIOutBufs = kN2 / kKc;               // one staging box per 32 output columns
constexpr int kIEpiWarp0 = 1;
constexpr int kIColWarp0 = kIEpiWarp0 + 4;
constexpr int kIThreads = (kIColWarp0 + 4 * kGroups) * 32;  // 416
constexpr int kIEpiSync = (3 << 10) | 128;         // named barrier 3 over the epilogue warps
constexpr int kIOffOut = 0;
constexpr int kIOffF = kIOffOut + kIOutBufs * kBoxBytes;
constexpr int kIOffCol = kIOffF + kIFBytes;
constexpr int kIOffTw = kIOffCol + kGroups * kColEntries * 8;
constexpr int kIOffBar = kIOffTw + kTwEntries * 8;
constexpr int kIBars = 2 * kIAStages + 2 * kIDStages;
constexpr int kISmemBytes = kIOffBar + kIBars * 8 + 16 + 1024;
static_assert(kISmemBytes <= 227 * 1024, "shared memory");
static_assert(kISmemBytes > 114 * 1024, "one CTA per SM: the CTA takes all of tensor memory");

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
                 "r"(tma::smem_addr(src)), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed bulk stores of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int G>
__device__ __forceinline__ bool inverse_column_group(const float2* __restrict__ modes, uint64_t* afull,
                                                     uint64_t* aempty, uint32_t tmem, float2* tile,
                                                     const float2* twc, long long nf, int m1, int m2)
{
    constexpr int kSync = ((1 + G) << 10) | 128;
    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int gt = tid - (kIColWarp0 + 4 * G) * 32;
    const int r = (warp & 3) * 32 + lane;
    const int cc = gt % kCW;
    const int ct = gt / kCW;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float2 zero = make_float2(0.0f, 0.0f);
    float2 next[CP::E];
    auto load = [&](long long i) {
        const long long f = static_cast<long long>(blockIdx.x) + i * gridDim.x;
        const float2* mf = modes + f * (2LL * m1 * m2);
#pragma unroll
        for (int e = 0; e < CP::E; ++e) {
            const int row = engine::mode_row(ct + e * CP::P, kN1, m1);
            next[e] = (i < nf && cc < m2 && row >= 0) ? __ldg(mf + row * m2 + cc) : zero;
        }
    };
    load(G);
    constexpr float kScale = 1.0f / (kN1 * kN2);  // a power of two: the scalings below are exact
    for (long long i = G; i < nf; i += kGroups) {
        float2 v[CP::E];
#pragma unroll
        for (int e = 0; e < CP::E; ++e) {
            v[e] = next[e];
        }
        load(i + kGroups);
        engine::run_passes<CP, true, 8, kCW, kSync>(v, ct, tile + cc, twc);
        // The last exchange's reads are done (its trailing barrier): the tile takes the result.
#pragma unroll
        for (int e = 0; e < CP::E; ++e) {
            const int row = ct + e * CP::P;
            tile[row * kCW + (cc ^ (row & 15))] = v[e];
        }
        engine::exchange_sync<1, kSync>();
        uint32_t hi[kIK], lo[kIK];
#pragma unroll
        for (int k = 0; k < kCW; ++k) {
            const float2 z = tile[r * kCW + (k ^ (r & 15))];
            const float c = k == 0 ? kScale : 2.0f * kScale;
            const float re = z.x * c;
            const float im = -z.y * c;
            const float hre = tf32_round(re);
            const float him = tf32_round(im);
            hi[k] = __float_as_uint(hre);
            lo[k] = __float_as_uint(tf32_round(re - hre));
            hi[kCW + k] = __float_as_uint(him);
            lo[kCW + k] = __float_as_uint(tf32_round(im - him));
        }
        engine::exchange_sync<1, kSync>();  // the tile's reads done before the next field's passes
        const int a = static_cast<int>(i % kIAStages);
        const bool ok = i < kIAStages || tma::mbar_wait(&aempty[a], static_cast<unsigned>(i / kIAStages - 1) & 1u);
        if (!group_all<(kSync >> 10)>(ok)) {
            return false;
        }
        fence_after_sync();
        const uint32_t acol = tmem + lane_base + kIACol0 + static_cast<uint32_t>(a) * kIACols;
        tmem_store32(acol, hi);
        tmem_store32(acol + kIK, lo);
        tmem_wait_store();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&afull[a]);
        }
    }
    return true;
}

__global__ void __launch_bounds__(kIThreads, 1)
    pruned_tc_inverse_kernel(const __grid_constant__ CUtensorMap map_y, const float2* __restrict__ modes,
                             long long fields, int m1, int m2, const float2* __restrict__ f_rows,
                             const float2* __restrict__ twc_g, unsigned* fault)
{
    allow_next_grid();
    extern __shared__ unsigned char smem_base[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_base) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* outs = smem + kIOffOut;
    unsigned char* fs = smem + kIOffF;
    auto* colbuf = reinterpret_cast<float2*>(smem + kIOffCol);
    auto* twc = reinterpret_cast<float2*>(smem + kIOffTw);
    auto* afull = reinterpret_cast<uint64_t*>(smem + kIOffBar);  // a field's A' stored (4 warps)
    uint64_t* aempty = afull + kIAStages;                          // its MMAs completed
    uint64_t* dfull = aempty + kIAStages;                          // a field's MMAs completed
    uint64_t* dempty = dfull + kIDStages;                          // its accumulator read (4 warps)
    auto* tmem_slot = reinterpret_cast<uint32_t*>(dempty + kIDStages);

    const int tid = static_cast<int>(threadIdx.x);
    const int warp = tid >> 5;
    const int lane = tid & 31;

    for (int i = tid; i < kIFBytes / 8; i += kIThreads) {
        reinterpret_cast<float2*>(fs)[i] = f_rows[i];
    }
    engine::fill_pass_twiddles<CP, true>(twc, twc_g);
    tma::fence_proxy_async();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tma::smem_addr(tmem_slot)),
                     "n"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int a = 0; a < kIAStages; ++a) {
            tma::mbar_init(&afull[a], 4);
            tma::mbar_init(&aempty[a], 1);
        }
        for (int d = 0; d < kIDStages; ++d) {
            tma::mbar_init(&dfull[d], 1);
            tma::mbar_init(&dempty[d], 4);
        }
        tma::fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // The set-up above reads only host-built tables and this CTA's own resources, so it overlaps
    // the previous kernel's tail; from here on global data another kernel may write is touched.
    wait_for_previous_grid();

    const long long bx = blockIdx.x;
    const long long nf = fields > bx ? (fields - 1 - bx) / gridDim.x + 1 : 0;
    bool failed = false;
    long long committed = 0;  // warp 0: fields whose MMAs were committed

    if (warp == 0) {
        const uint32_t f0 = tma::smem_addr(fs);
        for (long long i = 0; i < nf; ++i) {
            const uint32_t d = static_cast<uint32_t>(i % kIDStages);
            const int a = static_cast<int>(i % kIAStages);
            bool ok = i < kIDStages || tma::mbar_wait(&dempty[d], static_cast<unsigned>(i / kIDStages - 1) & 1u);
            ok = ok && tma::mbar_wait(&afull[a], static_cast<unsigned>(i / kIAStages) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                failed = true;
                break;
            }
            fence_after_sync();
            if (elect_one()) {
                const uint32_t dcol = tmem + d * kIDCols;
                const uint32_t acol = tmem + kIACol0 + static_cast<uint32_t>(a) * kIACols;
#pragma unroll
                for (int j = 0; j < kIK / 8; ++j) {
                    const uint32_t kstep = f0 + static_cast<uint32_t>(j * 2 * kILbo);
                    const uint64_t c_hi = f_desc_lbo<kILbo>(kstep);
                    const uint64_t c_lo = f_desc_lbo<kILbo>(kstep + kN2 / 8 * 128);
                    mma_ts(dcol, acol + 8 * j, c_hi, idesc(kN2), j > 0 ? 1u : 0u);  // x_hi C_hi
                    mma_ts(dcol, acol + 8 * j, c_lo, idesc(kN2), 1u);               // x_hi C_lo
                    mma_ts(dcol, acol + kIK + 8 * j, c_hi, idesc(kN2), 1u);         // x_lo C_hi
                }
                mma_commit(&aempty[a]);
                mma_commit(&dfull[d]);
            }
            __syncwarp();
            ++committed;
        }
    } else if (warp < kIColWarp0) {
        // Epilogue: thread = output row r of the field = TMEM lane r.
        const int et = tid - kIEpiWarp0 * 32;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        for (long long i = 0; i < nf; ++i) {
            const int d = static_cast<int>(i % kIDStages);
            const bool ok = tma::mbar_wait(&dfull[d], static_cast<unsigned>(i / kIDStages) & 1u);
            if (!group_all<(kIEpiSync >> 10)>(ok)) {
                failed = true;
                break;
            }
            fence_after_sync();
            const long long f = bx + i * gridDim.x;
#pragma unroll 1
            for (int c = 0; c < kIOutBufs; ++c) {
                if (et == 0) {
                    bulk_wait_read<kIOutBufs - 1>();  // box c of the previous field has left
                }
                engine::exchange_sync<1, kIEpiSync>();
                uint32_t v[32];
                tmem_load32(tmem + lane_base + static_cast<uint32_t>(d) * kIDCols + 32 * c, v);
                tmem_wait_load(v);
                if (c == kIOutBufs - 1) {
                    fence_before_sync();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&dempty[d]);
                    }
                }
                // Row r of the box at r * 128 bytes, 16-byte piece j at piece j ^ (r mod 8): the
                // TMA's 128-byte swizzle, and 8 distinct bank groups per quarter-warp.
                unsigned char* row = outs + c * kBoxBytes + r * 128;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) =
                        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
                tma::fence_proxy_async();
                engine::exchange_sync<1, kIEpiSync>();
                if (et == 0) {
                    tma_store_2d(&map_y, outs + c * kBoxBytes, c * kKc, static_cast<int>(f * kN1));
                    bulk_commit();
                }
            }
        }
        if (et == 0) {
            bulk_wait_all();
        }
    } else if (warp < kIColWarp0 + 4) {
        failed = !inverse_column_group<0>(modes, afull, aempty, tmem, colbuf, twc, nf, m1, m2);
    } else {
        failed = !inverse_column_group<1>(modes, afull, aempty, tmem, colbuf + kColEntries, twc, nf, m1, m2);
    }

    if (__syncthreads_or(failed)) {
        bool drained = true;
        if (tid == 0) {
            atomicOr(fault, tma::kFaultWaitTimeout);
            if (committed > 0) {
                const long long i = committed - 1;
                drained = tma::mbar_wait(&aempty[i % kIAStages], static_cast<unsigned>(i / kIAStages) & 1u);
            }
        }
        if (!drained) {
            atomicOr(fault, tma::kFaultDrainTimeout);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled encode_fn()
{
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess
            && q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
        }
    });
    if (fn == nullptr) {
        throw CudaError("rfft2_modes: cuTensorMapEncodeTiled is not available from the driver");
    }
    return fn;
}

}  // namespace

bool pruned_tc_fits(const void* x, int n1, int n2, int m1, int m2, long long fields)
{
    return n1 == kN1 && n2 == kN2 && m1 >= 1 && 2 * m1 <= kN1 && m2 >= 1 && m2 <= kMaxM2 && fields >= 1
           && fields <= INT_MAX / kN1 && (reinterpret_cast<unsigned long long>(x) & 15u) == 0;
}

namespace {

// A 2D tensor map over fields * 128 rows of 128 floats, boxes of 32 floats x 128 rows with the
// 128-byte swizzle.
CUtensorMap field_rows_map(const float* base, long long fields)
{
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kN2), static_cast<cuuint64_t>(fields) * kN1};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kN2) * sizeof(float)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kKc), static_cast<cuuint32_t>(kN1)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult res = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                                     strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (res != CUDA_SUCCESS) {
        throw CudaError("rfft2 modes: cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(res)) + ")");
    }
    return map;
}

}  // namespace

void pruned_tc_inverse(const float2* modes, float* y, int m1, int m2, long long fields, cudaStream_t stream)
{
    static std::atomic<bool> opted[kMaxDevices];
    const int device = current_device();
    if (!opted[device].load(std::memory_order_relaxed)) {
        SPECTRAL_CUDA(cudaFuncSetAttribute(pruned_tc_inverse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kISmemBytes));
        opted[device].store(true, std::memory_order_relaxed);
    }
    const float2* f_rows = twiddles::tf32_idft_rows(kN2);
    const float2* twc = twiddles::pass_table(kN1, CP::E);
    const CUtensorMap map = field_rows_map(y, fields);
    const long long sms = device_sm_count(device);
    const unsigned grid = static_cast<unsigned>(fields < sms ? fields : sms);
    launch_pdl(pruned_tc_inverse_kernel, dim3(grid), dim3(kIThreads), static_cast<std::size_t>(kISmemBytes), stream,
               map, modes, fields, m1, m2, f_rows, twc, device_fault_word());
}

void pruned_tc_forward(const float* x, float2* modes, int m1, int m2, long long fields, cudaStream_t stream)
{
    static std::atomic<bool> opted[kMaxDevices];
    const int device = current_device();
    if (!opted[device].load(std::memory_order_relaxed)) {
        SPECTRAL_CUDA(cudaFuncSetAttribute(pruned_tc_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes));
        opted[device].store(true, std::memory_order_relaxed);
    }
    const float2* f_rows = twiddles::tf32_dft_rows(kN2, m2);
    const float2* twc = twiddles::pass_table(kN1, CP::E);
    const CUtensorMap map = field_rows_map(x, fields);
    const long long sms = device_sm_count(device);
    const unsigned grid = static_cast<unsigned>(fields < sms ? fields : sms);
    launch_pdl(pruned_tc_forward_kernel, dim3(grid), dim3(kThreads), static_cast<std::size_t>(kSmemBytes), stream,
               map, modes, fields, m1, m2, f_rows, twc, device_fault_word());
}

}  // namespace spectral
