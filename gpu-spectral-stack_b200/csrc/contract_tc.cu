// The per-mode channel contraction on the 5th-generation tensor cores (tcgen05), in FP32
// accuracy through split TF32 ("3xTF32"):
//   out[b, o, m] = sum_i x[b, i, m] w[i, o, m]      (complex values)
//
// One mode is a complex GEMM (samples x outputs, summed over input channels). Written as one
// real GEMM per tile of 64 samples and T outputs,
//   D = A B^T,  A = [Re x ; Im x] (128 rows: samples x {re, im}, K = input channels),
//               B = [Re w | Im w] (2 T rows: outputs x {re, im}, K = input channels),
// D holds all four real products, and Re out = XrWr - XiWi, Im out = XrWi + XiWr are read off
// it. A row order that puts the re and im rows of one sample 16 lanes apart in TMEM lets one warp
// shuffle (xor 16) combine them in the epilogue.
//
// Precision: tcgen05 kind::tf32 multiplies 19-bit TF32 values. Each FP32 operand a is split into
// a_hi = tf32(a) (round to nearest) and a_lo = tf32(a - a_hi) (a - a_hi is exact in FP32); a product is a_hi b_hi +
// a_hi b_lo + a_lo b_hi, which keeps about 21 bits: the error of an FP32 dot product, not of a
// TF32 one. The tensor core rounds its FP32 accumulator once per MMA, so the large products
// a_hi b_hi go to one TMEM accumulator and the two small ones to another: the large sum takes
// one rounding per 8 channels instead of three, and the small sum's roundings are 2^-11 smaller.
// The epilogue adds the two in FP32 registers. The accumulator's rounding still grows with the
// number of channels (measured: within the FP32 tolerance 2 eps (log2 cin + 1) up to cin = 256,
// not beyond), so the entry point accepts cin up to 256 for this method.
//
// Data: the mode index is the fastest in x, w and out, so a CTA takes a group of G consecutive
// modes; G = 4 makes each (sample, channel) run one 32-byte sector. The CTA computes the G modes'
// 128 x 2T products with K = cin for one tile of 64 samples and T = 128 / G outputs (grid: mode
// groups x output tiles x sample tiles; a large and a small accumulator of 2T columns per mode
// fill the 512 TMEM columns). Warp roles:
//   - warp 0: the TMA loads of raw chunks of 8 input channels (x as [il][b][j], w as [il][o][j],
//     4 stages in flight) and, per chunk, the 3 G MMAs (G modes x 3 split products, M = 128,
//     N = 2T, K = 8), committed to the chunk's mbarrier; the warp runs converged, so its
//     descriptors are warp-uniform, and one elected lane issues;
//   - warps 1 ..: convert each raw chunk into the split operands in the canonical K-major,
//     unswizzled UMMA layout (core matrices of 8 rows x 16 bytes; two conversion stages), one
//     (row, mode) item per thread, then arrive on the stage's "converted" mbarrier;
//   - all warps, at the end: read the accumulators with tcgen05.ld, combine the real products,
//     stage the complex results per (sample, output) and store G x 8 bytes each.
// The warps meet only on mbarriers while the chunks stream, so the conversion of chunk c + 1,
// the MMAs of chunk c and the loads of the next chunks overlap. Every wait is bounded
// (tma.cuh); a wait that gives up records a fault code, the CTA drains what it issued (bounded),
// frees its TMEM and returns. The tensor maps cover this GPU's own x and w, and no load is
// multicast.

#include "../../include/spectral_b200.h"

#include "backend.hpp"
#include "launch.cuh"
#include "tma.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

namespace spectral {
namespace {

constexpr int kGroup = 4;          // modes per CTA (2 or 4)
constexpr int kKc = 8;             // input channels per chunk: one MMA K step (tf32: 32 bytes)
constexpr int kTileB = 64;         // samples per CTA (A rows = 2 kTileB = 128)
constexpr int kTileO = 128 / kGroup; // outputs per CTA (B rows = 2 kTileO; TMEM: kGroup x 2 x 2 kTileO = 512)
constexpr int kRows = 2 * kTileB;  // 128
constexpr int kCols = 2 * kTileO;  // D columns per accumulator
constexpr int kProducerWarps = (kTileB + kTileO) * kGroup / 32;  // one (row, mode) item per thread
constexpr int kThreads = 32 * (1 + kProducerWarps);
constexpr int kRawStages = 4;
constexpr int kConvStages = 2;
constexpr int kMaxCin = 256;       // the accuracy limit measured for this method

// Raw chunk (TMA box order, the mode innermost): x as [il][b][j], w as [il][o][j], complex.
constexpr int kRawXBytes = kKc * kTileB * kGroup * 8;
constexpr int kRawWBytes = kKc * kTileO * kGroup * 8;
constexpr int kRawBytes = kRawXBytes + kRawWBytes;
// Operand planes: rows x 8 TF32 in the canonical K-major layout without swizzle: the byte offset
// of (row r, k) is (k / 4) LBO + (r / 8) SBO + (r % 8) 16 + (k % 4) 4, SBO = 128 (8-row core-matrix
// groups back to back) and LBO = rows / 8 * 128 (the second 4-value half of K after the first).
constexpr int kSbo = 128;
constexpr int kLboA = (kRows / 8) * kSbo;  // 2 KiB
constexpr int kLboB = (kCols / 8) * kSbo;
constexpr int kPlaneA = kRows * kKc * 4;   // 4 KiB
constexpr int kPlaneB = kCols * kKc * 4;
// Per mode: A hi, A lo, B hi, B lo, plus 128 / kGroup bytes so that the modes' planes start on
// different banks (a quarter-warp's 16-byte stores, 8 / kGroup rows x kGroup modes, then never
// collide).
constexpr int kModeBytes = 2 * kPlaneA + 2 * kPlaneB + 128 / kGroup;
constexpr int kConvBytes = ((kGroup * kModeBytes + 1023) / 1024) * 1024;
constexpr int kPipeBytes = kRawStages * kRawBytes + kConvStages * kConvBytes;
constexpr int kBarBytes = 8 * (kRawStages + 2 * kConvStages) + 8;
constexpr int kSmemBytes = kPipeBytes + kBarBytes + 1024;  // + alignment slack for the 1 KiB base
constexpr int kTmemCols = kGroup * 2 * kCols;  // per mode a large and a small accumulator: 512
// Epilogue staging: out[b][o][j] complex, each b row padded by 16 bytes against bank conflicts.
constexpr int kStagePitch = kTileO * kGroup * 8 + 16;
static_assert(kTileB * kStagePitch <= kPipeBytes, "epilogue staging reuses the pipeline buffers");
static_assert(kSmemBytes <= 227 * 1024, "shared memory");

// The instruction descriptor of tcgen05.mma kind::tf32: F32 accumulator, TF32 A and B, both
// K-major, no negation, N = kCols, M = 128 (bits: c_format 4-5, a_format 7-9, b_format 10-12,
// n_dim = N / 8 at 17-22, m_dim = M / 16 at 24-28).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kCols / 8) << 17)
                            | (static_cast<uint32_t>(kRows / 16) << 24);

// Shared-memory matrix descriptor: start address, leading and stride byte offsets (all in
// 16-byte units), version 1 (Blackwell) at bit 46, no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, int lbo)
{
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16)
           | (static_cast<uint64_t>((kSbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// a rounded to TF32 (10 fraction bits), to nearest with ties away from zero: half a TF32 unit
// (bit 12) is added to the magnitude bits and the 13 low bits cleared. Two full-rate integer
// operations, where a conversion instruction runs at a fraction of that rate; the conversion's
// rounding for every finite input that does not round up to infinity (FFT data never does).
__device__ __forceinline__ float tf32_round(float a)
{
    return __uint_as_float((__float_as_uint(a) + 0x1000u) & 0xFFFFE000u);
}

// One 3D tiled TMA load of `map`'s box at coordinates (c0, c1, c2) into shared `dst`, completing
// on `bar`. The box's innermost extent is kGroup complex values (16 or 32 bytes), and c0 is a
// multiple of kGroup.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(tma::smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(tma::smem_addr(bar))
        : "memory");
}

// True in exactly one lane of the (converged) warp.
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

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
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

// 32 consecutive FP32 columns of this warp's 32 TMEM lanes, one lane per thread.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    // The loaded registers are in-out operands of the wait, so no use of them moves above it.
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] = __uint_as_float(r[i]);
    }
}

// Row of A (sample b, part 0 = re / 1 = im): 16 re rows, then the same 16 samples' im rows, per
// block of 32 (one warp's TMEM lanes).
__device__ __forceinline__ int a_row(int b, int part) { return (b >> 4) * 32 + part * 16 + (b & 15); }

// Byte offset of the 16-byte row segment (row r, channels 4 kh .. 4 kh + 3) in a plane.
template <int Lbo>
__device__ __forceinline__ uint32_t segment(int r, int kh)
{
    return static_cast<uint32_t>(kh * Lbo + (r >> 3) * kSbo + (r & 7) * 16);
}

// Splits 4 values into their TF32 hi and lo parts and stores each as one 16-byte segment.
__device__ __forceinline__ void put_split4(unsigned char* hi, unsigned char* lo, uint32_t off, float a0,
                                          float a1, float a2, float a3)
{
    const float4 h = make_float4(tf32_round(a0), tf32_round(a1), tf32_round(a2), tf32_round(a3));
    const float4 l = make_float4(tf32_round(a0 - h.x), tf32_round(a1 - h.y), tf32_round(a2 - h.z),
                                 tf32_round(a3 - h.w));
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
}

// Converts one raw item (8 channels of one complex row: sample or output, mode j) into the re
// and im rows of its plane pair: 8 loads of 8 bytes (a warp's loads are 256 contiguous bytes), 8
// stores of 16 bytes (a quarter-warp's stores hit 8 distinct 16-byte bank groups).
template <int Lbo, int PlaneBytes>
__device__ __forceinline__ void convert_item(const unsigned char* raw, int item_stride, int item,
                                             unsigned char* plane_hi, int re_row, int im_row)
{
    float2 v[kKc];
#pragma unroll
    for (int il = 0; il < kKc; ++il) {
        v[il] = *reinterpret_cast<const float2*>(raw + il * item_stride + item * 8);
    }
    unsigned char* plane_lo = plane_hi + PlaneBytes;
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) {
        const float2* q = v + 4 * kh;
        put_split4(plane_hi, plane_lo, segment<Lbo>(re_row, kh), q[0].x, q[1].x, q[2].x, q[3].x);
        put_split4(plane_hi, plane_lo, segment<Lbo>(im_row, kh), q[0].y, q[1].y, q[2].y, q[3].y);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    contract_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                       float2* __restrict__ out, int cin, int cout, long long modes, unsigned* fault)
{
    allow_next_grid();
    extern __shared__ unsigned char smem_base[];
    // 1 KiB alignment for the operand planes (the descriptors need 16 bytes; TMA 128).
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_base) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* raw = smem;
    unsigned char* conv = smem + kRawStages * kRawBytes;
    auto* raw_full = reinterpret_cast<uint64_t*>(smem + kPipeBytes);   // TMA bytes landed
    uint64_t* converted = raw_full + kRawStages;                          // 12 producer warps arrived
    uint64_t* consumed = converted + kConvStages;                         // the stage's MMAs completed
    auto* tmem_slot = reinterpret_cast<uint32_t*>(consumed + kConvStages);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int m0 = static_cast<int>(blockIdx.x) * kGroup;
    const int o0 = static_cast<int>(blockIdx.y) * kTileO;
    const int b0 = static_cast<int>(blockIdx.z) * kTileB;
    const int chunks = cin / kKc;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tma::smem_addr(tmem_slot)),
                     "n"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < kRawStages; ++s) {
            tma::mbar_init(&raw_full[s], 1);
        }
        for (int s = 0; s < kConvStages; ++s) {
            tma::mbar_init(&converted[s], kProducerWarps);
            tma::mbar_init(&consumed[s], 1);
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

    bool failed = false;
    int loaded = 0;  // chunks whose TMA loads warp 0 has issued
    if (warp == 0) {
        // The loads and the MMAs: the whole warp walks the chunks (so addresses and descriptors
        // stay warp-uniform), one elected lane issues.
        auto load = [&](int c) {
            ++loaded;
            const int s = c % kRawStages;
            unsigned char* dst = raw + s * kRawBytes;
            if (elect_one()) {
                tma::mbar_arrive_expect_tx(&raw_full[s], kRawBytes);
                tma_load_3d(dst, &map_x, m0, b0, c * kKc, &raw_full[s]);
                tma_load_3d(dst + kRawXBytes, &map_w, m0, o0, c * kKc, &raw_full[s]);
            }
            __syncwarp();
        };
        for (int c = 0; c < kRawStages && c < chunks; ++c) {
            load(c);
        }
        const uint32_t conv0 = tma::smem_addr(conv);
        for (int c = 0; c < chunks; ++c) {
            const int cs = c % kConvStages;
            if (!tma::mbar_wait(&converted[cs], static_cast<unsigned>(c / kConvStages) & 1u)) {
                failed = true;
                break;
            }
            // Chunk c's raw stage has been read by every producer: refill it.
            if (c + kRawStages < chunks) {
                load(c + kRawStages);
            }
            fence_after_sync();
            const uint32_t base = conv0 + static_cast<uint32_t>(cs * kConvBytes);
            const uint32_t acc = c > 0 ? 1u : 0u;
            if (elect_one()) {
#pragma unroll
                for (int j = 0; j < kGroup; ++j) {
                    const uint32_t ahi = base + static_cast<uint32_t>(j * kModeBytes);
                    const uint32_t alo = ahi + kPlaneA;
                    const uint32_t bhi = alo + kPlaneA;
                    const uint32_t blo = bhi + kPlaneB;
                    const uint32_t big = tmem + static_cast<uint32_t>(j * 2 * kCols);
                    const uint32_t small = big + kCols;
                    mma_tf32(big, smem_desc(ahi, kLboA), smem_desc(bhi, kLboB), acc);
                    mma_tf32(small, smem_desc(ahi, kLboA), smem_desc(blo, kLboB), acc);
                    mma_tf32(small, smem_desc(alo, kLboA), smem_desc(bhi, kLboB), 1u);
                }
                mma_commit(&consumed[cs]);
            }
            __syncwarp();
        }
    } else {
        // Producers: item p; x items (b = p / kGroup, j = p % kGroup) for p < kTileB kGroup, then
        // w items (o, j). A warp's items are 32 / kGroup rows x kGroup modes.
        const int p = tid - 32;
        const bool is_x = p < kTileB * kGroup;
        const int item = is_x ? p : p - kTileB * kGroup;
        const int r = item / kGroup;
        const int j = item % kGroup;
        for (int c = 0; c < chunks; ++c) {
            const int rs = c % kRawStages;
            const int cs = c % kConvStages;
            bool ok = tma::mbar_wait(&raw_full[rs], static_cast<unsigned>(c / kRawStages) & 1u);
            if (ok && c >= kConvStages) {
                ok = tma::mbar_wait(&consumed[cs], static_cast<unsigned>((c - kConvStages) / kConvStages) & 1u);
            }
            if (!ok) {
                failed = true;
                break;
            }
            const unsigned char* rx = raw + rs * kRawBytes;
            unsigned char* mode = conv + cs * kConvBytes + j * kModeBytes;
            if (is_x) {
                convert_item<kLboA, kPlaneA>(rx, kTileB * kGroup * 8, item, mode, a_row(r, 0), a_row(r, 1));
            } else {
                convert_item<kLboB, kPlaneB>(rx + kRawXBytes, kTileO * kGroup * 8, item, mode + 2 * kPlaneA, r,
                                             kTileO + r);
            }
            // The generic-proxy stores become visible to the tensor core's async proxy; one
            // arrival per warp once all its lanes have stored and fenced.
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&converted[cs]);
            }
        }
    }

    // Every warp waits for the last chunk's MMAs (its commit tracks all earlier ones).
    if (!failed && chunks > 0) {
        const int last = chunks - 1;
        failed = !tma::mbar_wait(&consumed[last % kConvStages], static_cast<unsigned>(last / kConvStages) & 1u);
    }
    if (__syncthreads_or(failed)) {
        if (tid == 0) {
            atomicOr(fault, tma::kFaultWaitTimeout);
            // Let the loads and MMAs this CTA issued finish (bounded) before its shared memory
            // and accumulators are released: the last kRawStages loads, and the last commit.
            bool drained = true;
            for (int c = loaded > kRawStages ? loaded - kRawStages : 0; c < loaded; ++c) {
                drained = tma::mbar_wait(&raw_full[c % kRawStages], static_cast<unsigned>(c / kRawStages) & 1u)
                          && drained;
            }
            if (chunks > 0) {
                const int last = chunks - 1;
                drained = tma::mbar_wait(&consumed[last % kConvStages], static_cast<unsigned>(last / kConvStages) & 1u)
                          && drained;
            }
            if (!drained) {
                atomicOr(fault, tma::kFaultDrainTimeout);
            }
        }
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
        if (warp == 0) {
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols) : "memory");
        }
        return;
    }
    fence_after_sync();

    // Epilogue. Warps 0-7: warp w reads TMEM lanes 32 (w % 4) .. + 31 (A rows: samples
    // 16 (w % 4) .. + 15, re in lanes 0-15, im in lanes 16-31) of modes (w / 4) kGroup / 2 ..
    // + kGroup / 2 - 1. Per 32 outputs the large and small accumulators are added; then lane l and
    // its partner l ^ 16, which hold the same sample's re and im rows, swap their products with
    // Im w (the upper kTileO columns).
    unsigned char* stage = smem;  // the pipeline buffers are free now
    if (warp < 8) {
        const int quad = warp & 3;
        const int part = lane >> 4;
        const int b = quad * 16 + (lane & 15);
        for (int jj = 0; jj < kGroup / 2; ++jj) {
            const int j = (warp >> 2) * (kGroup / 2) + jj;
            const uint32_t big =
                tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(j * 2 * kCols);
            for (int h = 0; h < kTileO / 32; ++h) {  // outputs 32 h .. 32 h + 31
                float w_re[32], w_im[32], t[32];
                tmem_load32(big + 32 * h, w_re);
                tmem_load32(big + kCols + 32 * h, t);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    w_re[i] += t[i];
                }
                tmem_load32(big + kTileO + 32 * h, w_im);
                tmem_load32(big + kCols + kTileO + 32 * h, t);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    w_im[i] += t[i];
                    const float other = __shfl_xor_sync(0xffffffffu, w_im[i], 16);
                    // re row: XrWr - XiWi; im row: XiWr + XrWi
                    const float v = part == 0 ? w_re[i] - other : w_re[i] + other;
                    const int o = 32 * h + i;
                    *reinterpret_cast<float*>(stage + b * kStagePitch + (o * kGroup + j) * 8 + part * 4) = v;
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols) : "memory");
    }
    // 64 samples x kTileO outputs x kGroup modes: 16-byte pieces (2 modes).
    constexpr int kPieces = kGroup / 2;
    for (int e = tid; e < kTileB * kTileO * kPieces; e += kThreads) {
        const int piece = e % kPieces;
        const int o = (e / kPieces) % kTileO;
        const int b = e / (kPieces * kTileO);
        const float4 v = *reinterpret_cast<const float4*>(stage + b * kStagePitch + (o * kGroup + 2 * piece) * 8);
        *reinterpret_cast<float4*>(out + (static_cast<long long>(b0 + b) * cout + o0 + o) * modes + m0 + 2 * piece) = v;
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
        throw CudaError("mode_contract: cuTensorMapEncodeTiled is not available from the driver");
    }
    return fn;
}

// A 3D map over complex values (8-byte elements, dims innermost first: modes, rows, channels)
// with the box {kGroup modes, box_rows, 8 channels}; strides in complex values.
CUtensorMap make_map(const void* base, unsigned long long modes, unsigned long long rows,
                     unsigned long long channels, unsigned long long row_stride, unsigned long long channel_stride,
                     unsigned box_rows)
{
    CUtensorMap map;
    const cuuint64_t dims[3] = {modes, rows, channels};
    const cuuint64_t strides[2] = {row_stride * 8, channel_stride * 8};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kGroup), box_rows, static_cast<cuuint32_t>(kKc)};
    const cuuint32_t elem[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_INT64, 3, const_cast<void*>(base), dims, strides,
                                   box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        throw CudaError("mode_contract: cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    }
    return map;
}

}  // namespace

// True when the tensor-core contraction takes this shape: whole tiles of 64 samples, kTileO
// outputs, kGroup modes and 8 input channels, at most 256 input channels, 16-byte aligned arrays, and every
// coordinate within the tensor maps' 32-bit range.
bool contract_tc_fits(const void* x, const void* w, const void* out, long long batch, int cin, int cout,
                      long long modes)
{
    const auto a16 = [](const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15u) == 0; };
    return batch > 0 && modes > 0 && batch % kTileB == 0 && cout % kTileO == 0 && cin % kKc == 0 && cin <= kMaxCin
           && modes % kGroup == 0 && a16(x) && a16(w) && a16(out) && modes <= 0x7fffffffLL && batch <= 0x7fffffffLL
           && cout / kTileO <= 65535 && batch / kTileB <= 65535;
}

void contract_tc(const float2* x, const float2* w, float2* out, long long batch, int cin, int cout,
                 long long modes, cudaStream_t stream)
{
    static std::atomic<bool> opted[kMaxDevices];
    const int device = current_device();
    if (!opted[device].load(std::memory_order_relaxed)) {
        SPECTRAL_CUDA(cudaFuncSetAttribute(contract_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        opted[device].store(true, std::memory_order_relaxed);
    }
    const auto m = static_cast<unsigned long long>(modes);
    // x (batch, cin, modes): box {kGroup modes, 64 samples, 8 channels}; w (cin, cout, modes):
    // box {kGroup modes, kTileO outputs, 8 channels}.
    const CUtensorMap map_x = make_map(x, m, static_cast<unsigned long long>(batch), static_cast<unsigned long long>(cin),
                                       static_cast<unsigned long long>(cin) * m, m, kTileB);
    const CUtensorMap map_w = make_map(w, m, static_cast<unsigned long long>(cout), static_cast<unsigned long long>(cin),
                                       m, static_cast<unsigned long long>(cout) * m, kTileO);
    const dim3 grid(static_cast<unsigned>(modes / kGroup), static_cast<unsigned>(cout / kTileO),
                    static_cast<unsigned>(batch / kTileB));
    launch_pdl(contract_tc_kernel, grid, dim3(kThreads), static_cast<std::size_t>(kSmemBytes), stream, map_x, map_w,
               out, cin, cout, modes, device_fault_word());
}

}  // namespace spectral
