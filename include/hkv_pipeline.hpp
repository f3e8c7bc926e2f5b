// hkv_pipeline.hpp -- C++ shim over hkv.h with the reference pipeline's names.
//
// higgs-audio.cpp keeps its KV slots in BackendRuntime (src/higgs_pipeline.cpp
// :357-403) and rents them with acquire_backend_kv_cache_slot (:1191-1208),
// returning a move-only ScopedBackendKvCacheSlot whose destructor releases the
// slot (:372-403, :1210-1220).  Errors are exceptions: std::runtime_error, and
// std::out_of_range for index errors (:1138-1140).  This header gives the
// pipeline the same names, ownership and exception types on top of the C ABI,
// so the call sites change only in the runtime object they pass.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "hkv.h"

namespace hkv_pipeline {

// Turns an hkv status into the reference's exception types.
inline void check(const hkv_engine *eng, int status, const char *what) {
    if (status == HKV_OK) {
        return;
    }
    std::string msg = std::string(what) + ": " +
                      (eng != nullptr ? hkv_last_error(eng) : hkv_status_string(status));
    if (status == HKV_ERR_RANGE) {
        throw std::out_of_range(msg);
    }
    throw std::runtime_error(msg);
}

// Owns one engine (one page pool on one GPU); replaces BackendRuntime's
// kv_cache_slots / kv_cache_slot_busy arena.
class PagedKvRuntime {
  public:
    explicit PagedKvRuntime(const hkv_config &cfg) {
        check(nullptr, hkv_engine_create(&cfg, &eng_), "hkv_engine_create");
    }
    ~PagedKvRuntime() {
        if (eng_ != nullptr) {
            hkv_engine_destroy(eng_);
        }
    }
    PagedKvRuntime(const PagedKvRuntime &) = delete;
    PagedKvRuntime &operator=(const PagedKvRuntime &) = delete;

    hkv_engine *engine() const { return eng_; }

  private:
    hkv_engine *eng_ = nullptr;
};

// Move-only lease of one slot, released on destruction.
class ScopedBackendKvCacheSlot {
  public:
    ScopedBackendKvCacheSlot() = default;
    ScopedBackendKvCacheSlot(hkv_engine *eng, int slot) : eng_(eng), slot_(slot) {}
    ScopedBackendKvCacheSlot(const ScopedBackendKvCacheSlot &) = delete;
    ScopedBackendKvCacheSlot &operator=(const ScopedBackendKvCacheSlot &) = delete;
    ScopedBackendKvCacheSlot(ScopedBackendKvCacheSlot &&o) noexcept : eng_(o.eng_), slot_(o.slot_) {
        o.eng_ = nullptr;
        o.slot_ = -1;
    }
    ScopedBackendKvCacheSlot &operator=(ScopedBackendKvCacheSlot &&o) noexcept {
        if (this != &o) {
            release();
            eng_ = o.eng_;
            slot_ = o.slot_;
            o.eng_ = nullptr;
            o.slot_ = -1;
        }
        return *this;
    }
    ~ScopedBackendKvCacheSlot() { release(); }

    void release() {
        if (eng_ != nullptr && slot_ >= 0) {
            hkv_slot_release(eng_, slot_);
        }
        eng_ = nullptr;
        slot_ = -1;
    }
    int slot() const { return slot_; }
    // cache.used of the reference
    int64_t used() const {
        int64_t u = 0;
        check(eng_, hkv_slot_len(eng_, slot_, &u), "hkv_slot_len");
        return u;
    }
    void set_used(int64_t u) { check(eng_, hkv_slot_set_len(eng_, slot_, u), "hkv_slot_set_len"); }
    void advance(int64_t n_tokens) {
        const int32_t s = slot_;
        check(eng_, hkv_slot_advance(eng_, 1, &s, n_tokens), "hkv_slot_advance");
    }

  private:
    hkv_engine *eng_ = nullptr;
    int slot_ = -1;
};

// acquire_backend_kv_cache_slot(runtime, capacity): `share` maps a published
// reference-prompt prefix (copy-on-write) when one exists.
inline ScopedBackendKvCacheSlot acquire_backend_kv_cache_slot(PagedKvRuntime &rt,
                                                              int64_t capacity,
                                                              const hkv_prefix_key *share = nullptr) {
    int32_t slot = -1;
    check(rt.engine(), hkv_slot_acquire(rt.engine(), capacity, share, &slot),
          "acquire_backend_kv_cache_slot");
    return ScopedBackendKvCacheSlot(rt.engine(), slot);
}

// Positions of build_reference_prompt_ids (:2507-2524) that depend only on
// the reference wav and its transcript, and so hold the same KV rows for
// every request using that reference: <|tts|>, [<|ref_text|>, transcript
// ids...], <|ref_audio|>, and one row per delayed reference-code frame.
inline int64_t reference_prefix_tokens(size_t ref_text_ids, int64_t delayed_ref_rows) {
    return 1 + (ref_text_ids > 0 ? 1 + static_cast<int64_t>(ref_text_ids) : 0) + 1 +
           delayed_ref_rows;
}

// Key under which such a prefix is published: 64-bit FNV-1a over the
// reference-code cache key (reference_code_cache_key, :1545-1551: model path,
// wav path, size, mtime) and the transcript token ids, with the prefix length.
inline hkv_prefix_key reference_prefix_key(const std::string &code_cache_key,
                                           const std::vector<int32_t> &ref_text_ids,
                                           int64_t delayed_ref_rows) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&h](const void *data, size_t n) {
        const unsigned char *p = static_cast<const unsigned char *>(data);
        for (size_t i = 0; i < n; ++i) {
            h ^= p[i];
            h *= 1099511628211ull;
        }
    };
    mix(code_cache_key.data(), code_cache_key.size());
    mix(ref_text_ids.data(), ref_text_ids.size() * sizeof(int32_t));
    mix(&delayed_ref_rows, sizeof(delayed_ref_rows));
    hkv_prefix_key key;
    key.hash = h;
    key.n_tokens = reference_prefix_tokens(ref_text_ids.size(), delayed_ref_rows);
    return key;
}

// One decode layer for all live slots (the per-layer block :5748-5786).
inline void decode_layer(PagedKvRuntime &rt, int layer, const std::vector<int32_t> &slots,
                         const float *q, const float *k, const float *v, float *out,
                         hkv_stream stream) {
    check(rt.engine(),
          hkv_decode_step(rt.engine(), layer, static_cast<int32_t>(slots.size()), slots.data(),
                          q, k, v, out, stream),
          "hkv_decode_step");
}

}  // namespace hkv_pipeline
