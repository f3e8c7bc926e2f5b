// Exercises include/hkv_pipeline.hpp against a host-only engine (no GPU):
// RAII release, move semantics, and the reference's exception types.
#include <cstdio>
#include <stdexcept>

#include "hkv_pipeline.hpp"

#define EXPECT(c)                                                        \
    do {                                                                 \
        if (!(c)) {                                                      \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #c); \
            return 1;                                                    \
        }                                                                \
    } while (0)

int main() {
    hkv_config cfg;
    hkv_config_default(&cfg);
    cfg.n_layers = 2;
    cfg.n_pages = 8;
    cfg.max_slots = 2;
    cfg.context_length = 1024;
    cfg.device = -1;  // bookkeeping only
    hkv_pipeline::PagedKvRuntime rt(cfg);
    hkv_pool_stats st{};
    {
        auto a = hkv_pipeline::acquire_backend_kv_cache_slot(rt, 32);
        EXPECT(a.slot() >= 0 && a.used() == 0);
        hkv_pool_stats_get(rt.engine(), &st);
        EXPECT(st.live_slots == 1 && st.reserved == 2);
        auto b = std::move(a);  // ownership moves, no double release
        EXPECT(a.slot() == -1 && b.slot() >= 0);
        bool range = false;
        try {
            b.set_used(5);  // beyond the written rows
        } catch (const std::out_of_range &) {
            range = true;
        }
        EXPECT(range);
        auto c = hkv_pipeline::acquire_backend_kv_cache_slot(rt, 0);
        bool full = false;
        try {
            auto d = hkv_pipeline::acquire_backend_kv_cache_slot(rt, 0);  // slot table full
        } catch (const std::out_of_range &) {
            return 2;  // must not be a range error
        } catch (const std::runtime_error &e) {
            full = std::string(e.what()).find("slots") != std::string::npos;
        }
        EXPECT(full);
        bool nodev = false;
        try {
            std::vector<int32_t> slots{b.slot()};
            hkv_pipeline::decode_layer(rt, 0, slots, nullptr, nullptr, nullptr, nullptr, nullptr);
        } catch (const std::runtime_error &) {
            nodev = true;
        }
        EXPECT(nodev);
    }
    hkv_pool_stats_get(rt.engine(), &st);
    EXPECT(st.live_slots == 0 && st.reserved == 0 && st.free_pages == 8);

    // prefix keys: same reference -> same key; another transcript -> another key
    const std::vector<int32_t> text{11, 12, 13};
    const hkv_prefix_key k1 = hkv_pipeline::reference_prefix_key("m\nref.wav\n100\n7", text, 40);
    const hkv_prefix_key k2 = hkv_pipeline::reference_prefix_key("m\nref.wav\n100\n7", text, 40);
    const hkv_prefix_key k3 = hkv_pipeline::reference_prefix_key("m\nref.wav\n100\n7", {11, 12}, 40);
    const hkv_prefix_key k4 = hkv_pipeline::reference_prefix_key("m\nother.wav\n100\n7", text, 40);
    EXPECT(k1.hash == k2.hash && k1.n_tokens == 1 + 1 + 3 + 1 + 40);
    EXPECT(k3.hash != k1.hash && k3.n_tokens == k1.n_tokens - 1);
    EXPECT(k4.hash != k1.hash);
    EXPECT(hkv_pipeline::reference_prefix_tokens(0, 5) == 7);

    // before anything is published under a key, acquiring with it gives an
    // empty slot (the caller then writes the prompt and publishes it)
    {
        auto first = hkv_pipeline::acquire_backend_kv_cache_slot(rt, k1.n_tokens + 8, &k1);
        EXPECT(first.used() == 0);
        hkv_pool_stats_get(rt.engine(), &st);
        EXPECT(st.prefixes == 0 && st.shared_pages == 0);
    }
    std::printf("shim ok\n");
    return 0;
}
