// The C++ mirror's expert-parallel plans (litemind::b200::ep_plan over
// lm_moe_ep_chunk_plan), host only: chunk plans tile each destination's send range in
// order and stack the receive buffer chunk after chunk; bad input throws.
#include <cstdint>
#include <random>
#include <vector>

#include "Expect.hpp"
#include "litemind_b200/MoeLayer.hpp"

using litemind::b200::ep_plan;
int main() {
    Expect expect("EpPlanTest");
    constexpr int32_t world = 4, experts = 32, local = experts / world;
    std::mt19937 gen(7);
    std::uniform_int_distribution<int32_t> dist(0, 9);
    std::vector<int32_t> send(experts), recv(experts);
    for (auto& v : send) v = dist(gen);
    for (auto& v : recv) v = dist(gen);
    const lm_ep_plan whole = ep_plan(world, send, recv);
    for (int32_t chunks : {1, 2, 3, 8}) {
        std::vector<lm_ep_plan> plans;
        for (int32_t k = 0; k < chunks; ++k) plans.push_back(ep_plan(world, send, recv, chunks, k));
        int32_t base = 0;
        for (const lm_ep_plan& p : plans) {
            expect(p.recv_offset[0] == base, "chunks stack in the receive buffer");
            base += p.n_recv;
        }
        expect(base == whole.n_recv, "chunks receive every row");
        for (int32_t d = 0; d < world; ++d) {
            int32_t pos = whole.send_offset[d];
            for (int32_t k = 0; k < chunks; ++k) {
                const int32_t lo = k * local / chunks, hi = (k + 1) * local / chunks;
                int32_t want = 0;
                for (int32_t e = lo; e < hi; ++e) want += send[static_cast<size_t>(d * local + e)];
                expect(plans[static_cast<size_t>(k)].send_offset[d] == pos, "send ranges in order");
                expect(plans[static_cast<size_t>(k)].send_count[d] == want, "send count of the chunk");
                pos += want;
            }
            expect(pos == whole.send_offset[d] + whole.send_count[d], "chunks send every row");
        }
    }
    bool threw = false;
    try {
        (void)ep_plan(world, send, recv, local + 1, 0);  // more chunks than local experts
    } catch (const litemind::b200::Error& e) {
        threw = e.status() == LM_ERR_INVALID_ARGUMENT;
    }
    expect(threw, "too many chunks is an error");
    return expect.finish();
}
