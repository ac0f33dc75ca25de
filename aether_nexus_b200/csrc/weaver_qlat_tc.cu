// weaver_qlat_tc.cu — q_latent = scale * q . K_dict on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory): the query
// projection onto the dictionary that the reference leaves to its caller
// (nexus-core/src/weaver.rs:142) and that the cold scores gather from
// (weaver_kernel.metal:170-190).
//
// One CTA per (128-atom tile, kv head g, group of sequences): a GEMM tile
//   D[atom][n] = sum_d K_dict[g][atom][d] * Q[n][d],   n = (sequence, query row)
// with M = 128 atoms (A operand: two or one 128 x 64 f16 TMA boxes, 128-byte
// swizzle, K-major), N = the query rows of up to 256 / RP sequences (RP < 16
// packed densely, else padded to 16; B operand: written into shared memory
// in the same swizzled K-major layout),
// K = head_dim in steps of 16.  One thread issues the MMAs and commits them
// to an mbarrier; every warp then reads its 32 atoms' accumulator lanes with
// tcgen05.ld, scales, and stores each atom's rows contiguously into the fp32
// q_latent [B][Hkv][A][RP].  The per-atom weights w that the scatter then
// accumulates into are cleared by a plain memset launched first.
//
// Every wait is bounded; a CTA whose MMA wait expired still waits (bounded)
// for its MMAs before it frees its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kTcThreads = 128;
constexpr uint32_t kTcMaxN = 256;          // query rows per MMA (the N of one tcgen05.mma)

// Shared-memory matrix descriptor of a K-major operand tile written with the
// 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart): start
// address / 16, leading byte offset 16 B (unused with this swizzle), stride
// byte offset 1024 B, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset: 16 B
    d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: 1024 B
    d |= static_cast<uint64_t>(1u) << 46;            // version
    d |= static_cast<uint64_t>(2u) << 61;            // 128-byte swizzle
    return d;
}

// Instruction descriptor of kind::f16 with f16 A and B, fp32 accumulate,
// both operands K-major, M x N.
__device__ __forceinline__ uint32_t f16_f32_idesc(uint32_t M, uint32_t N) {
    return (1u << 4)                 // D format: f32
           | (0u << 7) | (0u << 10)  // A, B format: f16
           | ((N >> 3) << 17)        // N / 8
           | ((M >> 4) << 24);       // M / 16
}

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 16 columns of fp32 from tensor memory: lane i of the warp gets
// its TMEM lane's 16 consecutive columns.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// rpc: the columns of one sequence (RP below 16, so several sequences share a
// 16-column MMA slice; RP rounded up to 16 above); spc: sequences per CTA;
// tmem_cols: tensor-memory columns to allocate (a power of two >= 32 and >= N)
template <int D>
__global__ void __launch_bounds__(kTcThreads) qlat_tc_kernel(const __grid_constant__ CUtensorMap tm_kdict, const RunArgs a,
                                                             uint32_t rpc, uint32_t spc, uint32_t tmem_cols) {
    constexpr uint32_t kBoxes = D / 64;
    constexpr uint32_t kABox = kAtomTile * 128;  // 128 atoms x 64 f16
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* atile = smem;                          // [kBoxes][128 atoms][128 B]
    uint8_t* btile = smem + kBoxes * kABox;         // [kBoxes][N rows][128 B]
    __shared__ __align__(8) uint64_t tma_bar;
    __shared__ __align__(8) uint64_t mma_bar;
    __shared__ uint32_t tmem_base;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t t = blockIdx.x, g = blockIdx.y, b0 = blockIdx.z * spc;
    const uint32_t nseq = min(spc, a.B - b0);
    const uint32_t N = (nseq * rpc + 15) / 16 * 16;  // multiple of 16, <= 256

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(&tma_bar, 1);
        mbar_init(&mma_bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    if (tid == 0) {
        mbar_arrive_expect_tx(&tma_bar, kBoxes * kABox);
        const int32_t y = static_cast<int32_t>(g * a.dict_row_stride + t * kAtomTile);
#pragma unroll
        for (uint32_t bx = 0; bx < kBoxes; ++bx) tma_load_2d(atile + bx * kABox, &tm_kdict, &tma_bar, bx * 64, y);
    }
    // B operand: query rows n = s * rpc + r (sequence b0 + s, row r of kv head
    // g: query token r / G, q head g * G + r % G); rows r >= R and columns
    // past the last sequence are zero.  Each thread writes 16-byte chunks
    // straight into the swizzled layout.
    for (uint32_t x = tid; x < N * (D / 8); x += kTcThreads) {
        const uint32_t n = x / (D / 8), chunk = x % (D / 8);
        const uint32_t s = n / rpc, r = n % rpc;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (s < nseq && r < a.R) {
            const uint32_t j = r / a.G, h = g * a.G + r % a.G;
            v = *reinterpret_cast<const uint4*>(a.q + ((static_cast<uint64_t>(b0 + s) * a.nq + j) * a.Hq + h) * D +
                                                chunk * 8);
        }
        *reinterpret_cast<uint4*>(btile + (chunk >> 3) * (N * 128) + swz128(n, chunk & 7)) = v;
    }
    fence_proxy_async_shared();  // generic writes of the B tile before the tensor cores read it
    __syncthreads();

    bool ok = true;
    if (tid == 0) {
        ok = mbar_wait(&tma_bar, 0, a.status, 40);
        if (ok) {
            tc_fence_after();
            const uint32_t idesc = f16_f32_idesc(128, N);
            uint32_t acc = 0;
#pragma unroll
            for (uint32_t bx = 0; bx < kBoxes; ++bx)
#pragma unroll
                for (uint32_t ks = 0; ks < 4; ++ks) {  // 4 steps of 16 f16 (32 B) inside a 128-byte row
                    const uint64_t ad = sw128_kmajor_desc(smem_u32(atile + bx * kABox) + ks * 32);
                    const uint64_t bd = sw128_kmajor_desc(smem_u32(btile + bx * (N * 128)) + ks * 32);
                    tc_mma_f16(tmem, ad, bd, idesc, acc);
                    acc = 1;
                }
        }
        tc_commit(&mma_bar);  // arrives once every MMA issued above has completed (at once if none)
        if (!ok) mbar_drain(&tma_bar, 0);  // an expired wait: let the tile's copy land before the CTA exits
    }
    __syncthreads();
    const bool done = mbar_wait(&mma_bar, 0, a.status, 41);
    tc_fence_after();

    // epilogue: warp w reads TMEM lanes 32w..32w+31 (atoms), 16 columns at a time
    const uint32_t atom = t * kAtomTile + warp * 32 + lane;
    const uint32_t tlane = tmem + ((warp * 32u) << 16);
    if (done) {
        for (uint32_t c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            tc_ld16(tlane + c0, v);  // all lanes of the warp take part
            if (atom >= a.A) continue;
            if (rpc >= 4) {
                // groups of 4 columns: 4 rows of one sequence, one 16-byte store
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                    const uint32_t n = c0 + i, s = n / rpc, r0 = n % rpc;
                    if (s >= nseq || r0 >= a.RP) continue;
                    float x[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) x[k] = (r0 + k < a.R) ? v[i + k] * a.scale : 0.0f;
                    *reinterpret_cast<float4*>(a.qlat + ((static_cast<uint64_t>(b0 + s) * a.Hkv + g) * a.A + atom) * a.RP + r0) =
                        make_float4(x[0], x[1], x[2], x[3]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t n = c0 + i, s = n / rpc, r = n % rpc;
                    if (s < nseq)
                        a.qlat[((static_cast<uint64_t>(b0 + s) * a.Hkv + g) * a.A + atom) * a.RP + r] =
                            r < a.R ? v[i] * a.scale : 0.0f;
                }
            }
        }
    } else if (tid == 0) {
        // an expired wait: the MMAs may still be running; give them (bounded)
        // time before the tensor memory is freed
        mbar_drain(&mma_bar, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
}

}  // namespace

// Columns per sequence (RP below 16 packed densely: RP is a power of two, so
// a sequence never straddles a 4-column store group; RP rounded up to 16
// above) and sequences per CTA: as many as fit N <= 256.
static void qlat_tc_shape(const RunArgs& a, uint32_t* rpc, uint32_t* spc) {
    *rpc = a.RP < 16 ? a.RP : ((a.RP + 15) / 16) * 16;
    *spc = kTcMaxN / *rpc;
    if (*spc > a.B) *spc = a.B;
    if (*spc == 0) *spc = 1;
}

size_t qlat_tc_smem_bytes(const RunArgs& a) {
    uint32_t rpc, spc;
    qlat_tc_shape(a, &rpc, &spc);
    const size_t n = (static_cast<size_t>(spc) * rpc + 15) / 16 * 16;
    return 1024 + (a.D / 64) * (kAtomTile * 128 + n * 128);
}

bool qlat_tc_supported(const RunArgs& a) {
    return (a.D == 64 || a.D == 128) && a.RP <= kTcMaxN && qlat_tc_smem_bytes(a) <= 227 * 1024;
}

cudaError_t launch_qlat_tc(const RunArgs& a, const CUtensorMap& tm_kdict, cudaStream_t s) {
    uint32_t rpc, spc;
    qlat_tc_shape(a, &rpc, &spc);
    uint32_t cols = 32;
    while (cols < (spc * rpc + 15) / 16 * 16) cols <<= 1;
    const size_t smem = qlat_tc_smem_bytes(a);
    dim3 grid(a.n_atom_tiles, a.Hkv, (a.B + spc - 1) / spc);
    cudaError_t e = cudaMemsetAsync(a.w, 0, sizeof(float) * a.B * a.Hkv * static_cast<size_t>(a.A) * a.RP, s);
    if (e != cudaSuccess) return e;
    if (a.D == 128) {
        e = cudaFuncSetAttribute(qlat_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        qlat_tc_kernel<128><<<grid, kTcThreads, smem, s>>>(tm_kdict, a, rpc, spc, cols);
    } else {
        e = cudaFuncSetAttribute(qlat_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        qlat_tc_kernel<64><<<grid, kTcThreads, smem, s>>>(tm_kdict, a, rpc, spc, cols);
    }
    return cudaGetLastError();
}

}  // namespace weaver
