// ref_ops_driver.cpp — runs the reference's own multihead_attention kernel
// (nexus-core/src/ops.metal:528-616, the whole ops.metal compiled unmodified
// as host C++ through oracle/msl_shim_ops) on the CPU.  TEST INFRASTRUCTURE
// ONLY: it pins the C restatement oracle_mha in oracle/weaver_oracle.c.
//
// Launch shape of the reference (ops.rs:433-460): grid (q_heads,
// num_queries) threadgroups of min(64, head_dim) threads.  Threadgroups run
// one at a time; each kernel thread is a host thread.
#include <barrier>
#include <cstdint>
#include <memory>
#include <thread>
#include <vector>

struct uint2 {
    unsigned int x, y;
};
enum class mem_flags { mem_none, mem_device, mem_threadgroup };

void multihead_attention(const _Float16* Q, const _Float16* K_cache, const _Float16* V_cache, _Float16* output,
                         const unsigned int& total_kv_len, const unsigned int& head_dim, const unsigned int& q_heads,
                         const unsigned int& kv_heads, const unsigned int& num_queries, uint2 tg_id, uint2 tid_2d,
                         uint2 tgs_2d);

namespace {
thread_local std::barrier<>* tl_bar = nullptr;
}

namespace metal {
void threadgroup_barrier(mem_flags) { tl_bar->arrive_and_wait(); }
float simd_shuffle_xor(float, unsigned short) { return 0.0f; }  // not used by multihead_attention
}  // namespace metal

extern "C" int ref_multihead_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                       uint16_t* out, uint32_t total_kv_len, uint32_t head_dim, uint32_t q_heads,
                                       uint32_t kv_heads, uint32_t num_queries) {
    // the kernel's score array holds 4096 positions (ops.metal:560)
    if (head_dim == 0 || kv_heads == 0 || q_heads % kv_heads || total_kv_len > 4096 || total_kv_len < num_queries)
        return -2;
    const unsigned tgs = head_dim < 64 ? head_dim : 64;
    for (unsigned qi = 0; qi < num_queries; ++qi) {
        for (unsigned h = 0; h < q_heads; ++h) {
            std::barrier<> bar(tgs);
            std::vector<std::thread> th;
            th.reserve(tgs);
            for (unsigned t = 0; t < tgs; ++t) {
                th.emplace_back([&, t] {
                    tl_bar = &bar;
                    multihead_attention(reinterpret_cast<const _Float16*>(q), reinterpret_cast<const _Float16*>(k_cache),
                                        reinterpret_cast<const _Float16*>(v_cache), reinterpret_cast<_Float16*>(out),
                                        total_kv_len, head_dim, q_heads, kv_heads, num_queries, uint2{h, qi},
                                        uint2{t, 0}, uint2{tgs, 1});
                });
            }
            for (auto& x : th) x.join();
        }
    }
    return 0;
}
