// weaver_distill_tc.cu — atom selection (nexus-core/src/distiller.rs:185-234)
// as a tokens x atoms GEMM on the 5th-generation tensor cores, with the CPU
// rule's result reproduced bit for bit.
//
// The rule: per (token, kv head g) row x, the dot with every atom of g's
// dictionary, summed in dimension order in fp32 from -0.0; the 4 largest by
// (score desc, index asc); coefficient = f16(score).
//
// One CTA per 128 rows of one kv head: tcgen05.mma with M = 128 rows (A
// operand, written swizzled into shared memory by the CTA), N = 256 atoms (B
// operand: dictionary tiles by TMA, 128-byte swizzle), K = 16, fp32
// accumulators in tensor memory, two of them so the MMAs of atom tile t+1 run
// while the epilogue reads tile t.  The epilogue keeps each row's 8 largest
// approximate scores s'.
//
// Exactness.  Each f16 x f16 product is exact in fp32; the tensor cores add
// them in their own order and precision, the CPU rule in dimension order.
// Both sums differ from the real sum by at most d * 2^-23 * sum_i |x_i D_ai|
// (d additions, each losing at most one ulp of a partial sum bounded by that
// sum, with round-to-nearest or truncation), and sum_i |x_i D_ai| <=
// |x|_2 |D_a|_2, so |s' - s| <= E with
//   E = 2^-13 * |x|_2 * max_a |D_a|_2  (>= 4 * 2 d 2^-23 |x|_2 |D_a|_2 at d <= 128)
// plus, should the tensor cores flush subnormal inputs, the terms they could
// drop: (sum of the row's subnormal |x_i|) * max |D| + (sum_i |x_i|) * (the
// largest subnormal |D|).
// Let s4 be the 4th largest exact score and T' the 4th largest s'.  At most
// 3 atoms have s > s4, so at most 3 have s' > s4 + E: T' <= s4 + E.  Every
// atom with s >= s4 (the top 4 and every atom tied with the 4th) has
// s' >= s4 - E >= T' - 2E.  So if the 8th largest s' is below T' - 2E, every
// atom that can enter the exact top 4 is among the row's 8 kept atoms; those
// at or above T' - 2E are re-scored exactly (dimension order, from -0.0) and
// the top 4 of them by (score desc, index asc) is the CPU rule's answer.  If
// E = 0 (a zero row or a zero dictionary) every score is +-0 and the answer
// is atoms 0..3, which the kept list holds (the scan visits atoms in index
// order and equal values do not displace earlier ones).  A row whose list
// does not certify (near-ties among more than 8 atoms, non-finite inputs) is
// finished by the whole CTA with the exact full scan.  An optional debug word
// records the largest |s' - s| / E seen on re-scored atoms.
//
// Rows come either from a row list (row i of head i % Hkv, the weaver_distill
// layout) or from hot blocks (block src[k] of the hot pool, its 16 tokens of
// head g; codes to block dst[k] of the cold pool: the migration).  Every wait
// is bounded; a CTA whose wait expired lets its copies and MMAs finish
// (bounded) before it frees its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kDtThreads = 256;      // 8 warps: producer, MMA, 2 dictionary-scan, 4 epilogue
constexpr uint32_t kDtRows = 128;         // M: rows per CTA
constexpr uint32_t kDtAtoms = 256;        // N: atoms per MMA tile
constexpr uint32_t kDtKeep = 8;           // approximate scores kept per row
constexpr float kDtErr = 1.0f / 8192.0f;  // E = kDtErr * |x|_2 * max |D_a|_2 + subnormal terms (see the header)

__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset 16 B (unused with this swizzle)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;    // 8-row groups 1024 B apart
    d |= static_cast<uint64_t>(1u) << 46;            // descriptor version
    d |= static_cast<uint64_t>(2u) << 61;            // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void dt_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void dt_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void dt_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void dt_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 columns of this warp's 32 TMEM lanes (one row per lane) into r; the
// caller waits with dt_wait_ld before reading r.
__device__ __forceinline__ void dt_ld32(uint32_t taddr, uint32_t r[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void dt_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool dt_ranks_before(float sa, uint32_t ia, float sb, uint32_t ib) {
    const bool na = isnan(sa), nb = isnan(sb);
    if (na != nb) return nb;
    if (!na && sa != sb) return sa > sb;
    return ia < ib;
}

// The CPU rule's dot: dimension order, fp32, from -0.0.  x is row r of the
// swizzled A tile; drow the atom's dictionary row.
template <int D>
__device__ __forceinline__ float exact_dot(const uint8_t* atile, uint32_t r, const __half* drow) {
    constexpr uint32_t kABox = kDtRows * 128;
    float s = -0.0f;
#pragma unroll 4
    for (uint32_t c = 0; c < D / 8; ++c) {
        const uint4 xr = *reinterpret_cast<const uint4*>(atile + (c >> 3) * kABox + swz128(r, c & 7));
        const uint4 dr = __ldg(reinterpret_cast<const uint4*>(drow) + c);
        float xf[8], df[8];
        h8_to_f8(xr, xf);
        h8_to_f8(dr, df);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = __fmaf_rn(xf[e], df[e], s);
    }
    return s;
}

// Sorted insertion of (v, a) into the descending list m/ix (v > m[7]); equal
// values keep the earlier (smaller) index first.
__device__ __forceinline__ void keep_insert(float m[kDtKeep], uint32_t ix[kDtKeep], float v, uint32_t a) {
#pragma unroll
    for (uint32_t j = 0; j < kDtKeep; ++j) {
        const bool sw = v > m[j];
        const float tm = m[j];
        const uint32_t ti = ix[j];
        m[j] = sw ? v : tm;
        ix[j] = sw ? a : ti;
        v = sw ? tm : v;
        a = sw ? ti : a;
    }
}

// Offer 32 approximate scores (atoms a0 .. a0 + 31) to the kept list.  The
// values above the list's smallest go through the lane's row of shared
// memory and one rolled insertion loop: the insertion code exists once, not
// once per value (an unrolled copy per value made the loop's code larger than
// the instruction cache and every pass slow).
__device__ __forceinline__ void scan32(const uint32_t r[32], uint32_t a0, uint32_t A, float* row, float m[kDtKeep],
                                       uint32_t ix[kDtKeep]) {
    const float thr = m[kDtKeep - 1];
    uint32_t mask = 0;
#pragma unroll
    for (uint32_t i = 0; i < 32; i += 4) {
        *reinterpret_cast<float4*>(row + i) = make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                                                          __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) mask |= (__uint_as_float(r[i + e]) > thr ? 1u : 0u) << (i + e);
    }
    if (a0 + 32 > A) mask &= a0 >= A ? 0u : (1u << (A - a0)) - 1u;
#pragma unroll 1
    while (mask) {
        const uint32_t i = __ffs(mask) - 1;
        mask &= mask - 1;
        const float v = row[i];
        if (v > m[kDtKeep - 1]) keep_insert(m, ix, v, a0 + i);
    }
}

__device__ __forceinline__ uint4 pack_code(const uint32_t bi[4], const float bs[4], uint32_t nb) {
    uint16_t oi[4] = {0, 0, 0, 0}, oc[4] = {0, 0, 0, 0};
    for (uint32_t k = 0; k < nb && k < 4; ++k) {
        oi[k] = static_cast<uint16_t>(bi[k]);
        oc[k] = __half_as_ushort(__float2half_rn(bs[k]));
    }
    uint4 code;
    code.x = oi[0] | (static_cast<uint32_t>(oi[1]) << 16);
    code.y = oi[2] | (static_cast<uint32_t>(oi[3]) << 16);
    code.z = oc[0] | (static_cast<uint32_t>(oc[1]) << 16);
    code.w = oc[2] | (static_cast<uint32_t>(oc[3]) << 16);
    return code;
}

// Insertion of (s, a) into a running exact top 4 (dt_ranks_before order).
__device__ __forceinline__ void top4_insert(float bs[4], uint32_t bi[4], uint32_t& nb, float s, uint32_t a) {
    uint32_t pos = nb;
    while (pos > 0 && dt_ranks_before(s, a, bs[pos - 1], bi[pos - 1])) --pos;
    if (pos < 4) {
        for (uint32_t q = (nb < 4 ? nb : 3); q > pos; --q) {
            bs[q] = bs[q - 1];
            bi[q] = bi[q - 1];
        }
        bs[pos] = s;
        bi[pos] = a;
        if (nb < 4) ++nb;
    }
}

template <int D>
__global__ void __launch_bounds__(kDtThreads, 1)
    distill_tc_kernel(const __grid_constant__ CUtensorMap tm_dict, const DistillTcArgs p) {
    constexpr uint32_t kBoxes = D / 64;
    constexpr uint32_t kABox = kDtRows * 128;   // 128 rows x 64 f16
    constexpr uint32_t kBBox = kDtAtoms * 128;  // 256 atoms x 64 f16
    constexpr uint32_t kStage = kBoxes * kBBox;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* atile = smem;                       // [kBoxes][128 rows][128 B]
    uint8_t* btile = smem + kBoxes * kABox;      // [2 stages][kBoxes][256 atoms][128 B]
    __shared__ __align__(8) uint64_t full[2], empty[2], accf[2], acce[2], fin;
    __shared__ uint32_t tmem_base, s_dmax, s_dsub, s_dnorm2, n_fb;
    __shared__ float s_l1[kDtRows], s_l1sub[kDtRows], s_l2[kDtRows];
    __shared__ uint32_t s_out[kDtRows];          // output record of each row (~0u: no row)
    __shared__ uint32_t s_fb[kDtRows];           // rows left to the exact scan
    __shared__ float s_bs[kDtThreads / 32][4];
    __shared__ uint32_t s_bi[kDtThreads / 32][4], s_nb[kDtThreads / 32];
    __shared__ __align__(16) float s_stage[kDtRows][36];  // epilogue: one row of 32 scores per lane (padded)

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t g = blockIdx.y, tile = blockIdx.x;
    const uint32_t A = p.A, NT = (A + kDtAtoms - 1) / kDtAtoms;
    const __half* dict_g = p.dict + static_cast<uint64_t>(g) * p.dict_head_stride;
    uint32_t* status = p.diag + 2;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 3);  // the MMAs' commit + the two dictionary-scan warps
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], 4);   // one arrival per epilogue warp
        }
        mbar_init(&fin, 1);
        s_dmax = 0;
        s_dsub = 0;
        s_dnorm2 = 0;
        n_fb = 0;
        fence_barrier_init();
    }
    // A tile: row k of this CTA, 16-byte chunks straight into the swizzled
    // layout; each row's |x|_1 and output record
    for (uint32_t x = tid; x < kDtRows * (D / 8); x += kDtThreads) {
        const uint32_t k = x / (D / 8), c = x % (D / 8);
        const __half* src = nullptr;
        uint32_t outi = ~0u;
        if (p.src_blocks) {
            const uint32_t slot = tile * (kDtRows / kBlock) + k / kBlock;
            if (slot < p.n_blocks) {
                const uint32_t sb = p.src_blocks[slot], db = p.dst_blocks[slot];
                if (sb < p.src_limit && db < p.dst_limit) {
                    src = p.pool + ((static_cast<uint64_t>(sb) * kBlock + k % kBlock) * p.Hkv + g) * D;
                    outi = (db * kBlock + k % kBlock) * p.Hkv + g;
                } else if (c == 0 && k % kBlock == 0) {
                    atomicOr(p.bad, 1u);
                }
            }
        } else {
            const uint64_t ridx = g + static_cast<uint64_t>(p.Hkv) * (static_cast<uint64_t>(tile) * kDtRows + k);
            if (ridx < p.n_rows) {
                src = p.rows + ridx * D;
                outi = static_cast<uint32_t>(ridx);
            }
        }
        const uint4 v = src ? *reinterpret_cast<const uint4*>(src + c * 8) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(atile + (c >> 3) * kABox + swz128(k, c & 7)) = v;
        float f[8];
        h8_to_f8(v, f);
        float l1 = 0.0f, l1sub = 0.0f, l2 = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float a = fabsf(f[e]);
            l1 += a;
            l1sub += a < 6.103515625e-05f ? a : 0.0f;  // below the smallest normal f16
            l2 = __fmaf_rn(a, a, l2);
        }
        // a row's D/8 chunks sit in D/8 consecutive lanes (D/8 divides 32)
#pragma unroll
        for (uint32_t o = 1; o < D / 8; o <<= 1) {
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
            l1sub += __shfl_xor_sync(0xffffffffu, l1sub, o);
            l2 += __shfl_xor_sync(0xffffffffu, l2, o);
        }
        if (c == 0) {
            s_l1[k] = l1;
            s_l1sub[k] = l1sub;
            s_l2[k] = l2;
            s_out[k] = outi;
        }
    }
    fence_proxy_async_shared();  // generic writes of the A tile before the tensor cores read it
    __syncthreads();
    dt_fence_after();
    const uint32_t tmem = tmem_base;
    bool ok = true;
    float m[kDtKeep];      // epilogue: the row's largest approximate scores, descending
    uint32_t ix[kDtKeep];  // and their atoms
#pragma unroll
    for (uint32_t j = 0; j < kDtKeep; ++j) {
        m[j] = -INFINITY;
        ix[j] = 0;
    }

    if (warp == 0) {
        // ---- producer: dictionary tiles of 256 atoms
        if (lane == 0) {
            prefetch_tensormap(&tm_dict);
            uint32_t t = 0;
            for (; t < NT; ++t) {
                const uint32_t s = t & 1u;
                if (t >= 2 && !mbar_wait(&empty[s], ((t >> 1) - 1) & 1, status, 50)) break;
                mbar_arrive_expect_tx(&full[s], kStage);
                const int32_t y = static_cast<int32_t>(g * p.dict_row_stride + t * kDtAtoms);
#pragma unroll
                for (uint32_t bx = 0; bx < kBoxes; ++bx)
                    tma_load_2d(btile + s * kStage + bx * kBBox, &tm_dict, &full[s], bx * 64, y);
            }
            // the last copy into each stage has landed before the CTA exits
            for (uint32_t s = 0; s < 2 && s < t; ++s) mbar_drain(&full[s], (((t - s + 1) / 2) - 1) & 1);
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((kDtAtoms >> 3) << 17) | ((kDtRows >> 4) << 24);
            for (uint32_t t = 0; t < NT; ++t) {
                const uint32_t s = t & 1u;
                if (!mbar_wait(&full[s], (t >> 1) & 1, status, 51)) break;
                if (t >= 2 && !mbar_wait(&acce[s], ((t >> 1) - 1) & 1, status, 52)) break;
                dt_fence_after();
                uint32_t acc = 0;
#pragma unroll
                for (uint32_t bx = 0; bx < kBoxes; ++bx)
#pragma unroll
                    for (uint32_t ks = 0; ks < 4; ++ks) {
                        const uint64_t ad = sw128_desc(smem_u32(atile + bx * kABox) + ks * 32);
                        const uint64_t bd = sw128_desc(smem_u32(btile + s * kStage + bx * kBBox) + ks * 32);
                        dt_mma(tmem + s * kDtAtoms, ad, bd, idesc, acc);
                        acc = 1;
                    }
                dt_commit(&empty[s]);
                dt_commit(&accf[s]);
            }
            // every MMA issued above has completed before tensor memory is freed
            dt_commit(&fin);
            mbar_drain(&fin, 0);
        }
    } else if (warp < 4) {
        // ---- dictionary scan: max |D| over the head's atoms as 16-bit
        // magnitudes (an infinity or NaN shows as >= 0x7C00), and the largest
        // subnormal magnitude (below 0x0400)
        // and the largest squared atom norm (fp32 sums of exact squares; a
        // non-finite norm makes E non-finite)
        const uint32_t ht = tid - 64;
        uint32_t mx = 0, ms = 0;
        float n2 = 0.0f;
        for (uint32_t t = 0; t < NT; ++t) {
            const uint32_t s = t & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (t >> 1) & 1, status, 53))) break;
            const uint32_t rows = min(kDtAtoms, A - t * kDtAtoms);
            for (uint32_t row = ht; row < rows; row += 64) {
                float sq = 0.0f;
#pragma unroll
                for (uint32_t bx = 0; bx < kBoxes; ++bx)
#pragma unroll
                    for (uint32_t c = 0; c < 8; ++c) {
                        const uint4 v = *reinterpret_cast<const uint4*>(btile + s * kStage + bx * kBBox + swz128(row, c));
                        const uint32_t u[4] = {v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu, v.z & 0x7FFF7FFFu,
                                               v.w & 0x7FFF7FFFu};
                        float f[8];
                        h8_to_f8(v, f);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            mx = __vmaxu2(mx, u[j]);
                            ms = __vmaxu2(ms, u[j] & __vcmpltu2(u[j], 0x04000400u));
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) sq = __fmaf_rn(f[e], f[e], sq);
                    }
                n2 = (n2 != n2 || sq != sq) ? __int_as_float(0x7FC00000) : fmaxf(n2, sq);  // a NaN norm stays NaN
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        atomicMax(&s_dmax, max(mx & 0xFFFFu, mx >> 16));
        atomicMax(&s_dsub, max(ms & 0xFFFFu, ms >> 16));
        // non-negative floats (and +inf, NaN above them) order like their bits
        atomicMax(&s_dnorm2, __float_as_uint(n2));
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31, one row per lane
        const uint32_t q = warp & 3u;
        float* stage = s_stage[q * 32 + lane];
        for (uint32_t t = 0; t < NT; ++t) {
            const uint32_t s = t & 1u;
            ok = __all_sync(0xffffffffu, mbar_wait(&accf[s], (t >> 1) & 1, status, 54));
            if (!ok) break;
            dt_fence_after();
            const uint32_t taddr = tmem + ((q * 32u) << 16) + s * kDtAtoms;
            const uint32_t a0 = t * kDtAtoms;
            uint32_t va[32], vb[32];
            dt_ld32(taddr, va);
            dt_wait_ld();
#pragma unroll 1
            for (uint32_t c = 0; c < kDtAtoms; c += 64) {
                dt_ld32(taddr + c + 32, vb);  // in flight while va is scanned
                scan32(va, a0 + c, A, stage, m, ix);
                dt_wait_ld();
                if (c + 64 < kDtAtoms) dt_ld32(taddr + c + 64, va);
                scan32(vb, a0 + c + 32, A, stage, m, ix);
                dt_wait_ld();
            }
            dt_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[s]);
        }
    }
    dt_fence_before();
    __syncthreads();  // every role done: s_dmax final, the accumulators read, the MMAs complete

    if (warp >= 4) {
        // certify the kept list and re-score its candidates, or leave the row to the exact scan
        const uint32_t r = (warp & 3u) * 32 + lane;
        const uint32_t outi = s_out[r];
        if (outi != ~0u && ok && !timed_out(status)) {
            const float dmax = __half2float(__ushort_as_half(static_cast<unsigned short>(s_dmax)));
            const float dsub = __half2float(__ushort_as_half(static_cast<unsigned short>(s_dsub)));
            const float dn2 = __uint_as_float(s_dnorm2);
            // 17/16: room for the rounding of the norms, these products and the threshold below
            const float E = 1.0625f * (kDtErr * sqrtf(s_l2[r]) * sqrtf(dn2) + s_l1sub[r] * dmax + s_l1[r] * dsub);
            bool cert;
            float thr;
            if (E == 0.0f) {  // a zero row or dictionary: every score is +-0
                cert = m[3] > -INFINITY;
                thr = m[3];
            } else {
                thr = m[3] - 2.0f * E;
                cert = m[kDtKeep - 1] < thr;  // false for a NaN or infinite E or m
            }
            if (cert) {
                float bs[4];
                uint32_t bi[4], nb = 0;
#pragma unroll
                for (uint32_t j = 0; j < kDtKeep; ++j) {
                    if (!(m[j] >= thr)) continue;
                    const float sx = exact_dot<D>(atile, r, dict_g + static_cast<uint64_t>(ix[j]) * D);
                    top4_insert(bs, bi, nb, sx, ix[j]);
                    if (E > 0.0f) {
                        const float ratio = fabsf(m[j] - sx) / E;
                        atomicMax(p.diag, __float_as_uint(ratio));
                    }
                }
                p.out[outi] = pack_code(bi, bs, nb);
            } else {
                s_fb[atomicAdd(&n_fb, 1u)] = r;
            }
        }
    }
    __syncthreads();
    const uint32_t nfb = n_fb;
    if (tid == 0 && nfb) atomicAdd(p.diag + 1, nfb);
    // the exact full scan of the rows that did not certify: every thread takes
    // atoms tid, tid + 256, ...; warp and CTA merges of the per-thread top 4
    for (uint32_t f = 0; f < nfb; ++f) {
        const uint32_t r = s_fb[f];
        float bs[4];
        uint32_t bi[4], nb = 0;
        for (uint32_t a = tid; a < A; a += kDtThreads)
            top4_insert(bs, bi, nb, exact_dot<D>(atile, r, dict_g + static_cast<uint64_t>(a) * D), a);
        uint32_t head = 0, wn = 0;
        for (int k = 0; k < 4; ++k) {
            const bool have = head < nb;
            float cs = have ? bs[head] : 0.0f;
            uint32_t ci = have ? bi[head] : 0xFFFFFFFFu, cl = have ? lane : 0xFFFFFFFFu;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float os = __shfl_xor_sync(0xffffffffu, cs, off);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, ci, off);
                const uint32_t ol = __shfl_xor_sync(0xffffffffu, cl, off);
                const bool take = ol != 0xFFFFFFFFu && (cl == 0xFFFFFFFFu || dt_ranks_before(os, oi, cs, ci));
                if (take) {
                    cs = os;
                    ci = oi;
                    cl = ol;
                }
            }
            if (cl == 0xFFFFFFFFu) break;
            if (lane == 0) {
                s_bs[warp][k] = cs;
                s_bi[warp][k] = ci;
            }
            ++wn;
            if (lane == cl) ++head;
        }
        if (lane == 0) s_nb[warp] = wn;
        __syncthreads();
        if (tid == 0) {
            float fs[4];
            uint32_t fi[4], fnb = 0;
            for (uint32_t w = 0; w < kDtThreads / 32; ++w)
                for (uint32_t k = 0; k < s_nb[w]; ++k) top4_insert(fs, fi, fnb, s_bs[w][k], s_bi[w][k]);
            p.out[s_out[r]] = pack_code(fi, fs, fnb);
        }
        __syncthreads();
    }
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
}

// Scratch of calls that pass no diagnostics buffer: [max error ratio bits,
// rows left to the exact scan, status, first expired wait]; cleared before
// each such launch.
__device__ uint32_t g_dt_diag[4];

}  // namespace

size_t distill_tc_smem_bytes(uint32_t D) {
    return 1024 + (D / 64) * (static_cast<size_t>(kDtRows) * 128 + 2 * static_cast<size_t>(kDtAtoms) * 128);
}

bool distill_tc_supported(uint32_t D, uint32_t A, uint64_t dict_head_stride) {
    return (D == 64 || D == 128) && A >= 4 && A <= 65536 && dict_head_stride % D == 0;
}

cudaError_t launch_distill_tc(DistillTcArgs p, uint32_t D, const CUtensorMap& tm_dict, cudaStream_t s) {
    uint64_t rows_per_head;
    if (p.src_blocks) {
        rows_per_head = static_cast<uint64_t>(p.n_blocks) * kBlock;
    } else {
        rows_per_head = (p.n_rows + p.Hkv - 1) / p.Hkv;
    }
    if (rows_per_head == 0) return cudaSuccess;
    cudaError_t e;
    if (!p.diag) {
        void* d = nullptr;
        if ((e = cudaGetSymbolAddress(&d, g_dt_diag)) != cudaSuccess) return e;
        if ((e = cudaMemsetAsync(d, 0, sizeof(g_dt_diag), s)) != cudaSuccess) return e;
        p.diag = static_cast<uint32_t*>(d);
    }
    const size_t smem = distill_tc_smem_bytes(D);
    dim3 grid(static_cast<uint32_t>((rows_per_head + kDtRows - 1) / kDtRows), p.Hkv);
    if (D == 128) {
        e = cudaFuncSetAttribute(distill_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        distill_tc_kernel<128><<<grid, kDtThreads, smem, s>>>(tm_dict, p);
    } else {
        e = cudaFuncSetAttribute(distill_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        distill_tc_kernel<64><<<grid, kDtThreads, smem, s>>>(tm_dict, p);
    }
    return cudaGetLastError();
}

}  // namespace weaver
