// ref_driver.cpp — runs the reference's own weaver_decode kernel source
// (nexus-core/src/weaver_kernel.metal:118-240, compiled unmodified as host C++
// through oracle/msl_shim) on the CPU.  TEST INFRASTRUCTURE ONLY: the library
// it builds (oracle/_ref/libweaver_ref.so) pins the C restatement in
// oracle/weaver_oracle.c and generates tests/golden fixtures.
//
// Launch shape of the reference (weaver.rs:222-224): grid (1, q_heads, 1)
// threadgroups of 32 threads, one SIMD group per query head.  Here every
// lane is a host thread; the lanes of one head meet in simd_shuffle_xor.
#include <barrier>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

// Mirrors of the kernel's own types (weaver_kernel.metal:34-51); the layouts
// and names must match for the C++ symbol to link.
struct SparseCode {
    unsigned short indices[4];
    _Float16 coeffs[4];
};
struct WeaverParams {
    unsigned int q_heads, kv_heads, head_dim, block_size, gqa_group;
    unsigned int hot_count, cold_count, dict_size, sparsity_k;
    unsigned int _pad[3];
};
struct uint3 {
    unsigned int x, y, z;
};
static_assert(sizeof(SparseCode) == 16, "SparseCode is 16 bytes");
static_assert(sizeof(WeaverParams) == 48, "WeaverParams is 48 bytes");

// The reference kernel, as compiled from weaver_kernel.metal.
void weaver_decode(const _Float16* q_exact, const _Float16* q_latent, const _Float16* hot_pool,
                   const SparseCode* cold_pool, const unsigned int* loom_refs, _Float16* output,
                   WeaverParams& p, const _Float16* dictionary, uint3 gid, unsigned int tid);

namespace {
struct SimdGroup {
    float slots[32];
    std::barrier<> bar{32};
};
thread_local SimdGroup* tl_group = nullptr;
thread_local unsigned tl_lane = 0;
}  // namespace

namespace metal {
float simd_shuffle_xor(float value, unsigned short mask) {
    tl_group->slots[tl_lane] = value;
    tl_group->bar.arrive_and_wait();
    const float r = tl_group->slots[(tl_lane ^ mask) & 31u];
    tl_group->bar.arrive_and_wait();
    return r;
}
}  // namespace metal

// The kernel hard-codes HEAD_DIM = 128 and DICT_SIZE = 512
// (weaver_kernel.metal:23-26); other geometries are refused.
extern "C" int ref_weaver_decode(const uint16_t* q_exact, const uint16_t* q_latent,
                                 const uint16_t* hot_pool, const void* cold_pool,
                                 const uint32_t* loom_refs, const uint16_t* dictionary,
                                 const void* params, uint16_t* out) {
    WeaverParams p;
    std::memcpy(&p, params, sizeof(p));
    if (p.head_dim != 128 || p.dict_size != 512 || p.gqa_group == 0) return -2;
    const unsigned heads_per_wave = 8;
    for (unsigned h0 = 0; h0 < p.q_heads; h0 += heads_per_wave) {
        const unsigned nh = (p.q_heads - h0) < heads_per_wave ? (p.q_heads - h0) : heads_per_wave;
        std::vector<SimdGroup> groups(nh);
        std::vector<std::thread> lanes;
        lanes.reserve(nh * 32);
        for (unsigned hh = 0; hh < nh; ++hh) {
            for (unsigned lane = 0; lane < 32; ++lane) {
                lanes.emplace_back([&, hh, lane] {
                    tl_group = &groups[hh];
                    tl_lane = lane;
                    WeaverParams local = p;
                    weaver_decode(reinterpret_cast<const _Float16*>(q_exact),
                                  reinterpret_cast<const _Float16*>(q_latent),
                                  reinterpret_cast<const _Float16*>(hot_pool),
                                  static_cast<const SparseCode*>(cold_pool), loom_refs,
                                  reinterpret_cast<_Float16*>(out), local,
                                  reinterpret_cast<const _Float16*>(dictionary),
                                  uint3{lane, h0 + hh, 0}, lane);
                });
            }
        }
        for (auto& t : lanes) t.join();
    }
    return 0;
}
