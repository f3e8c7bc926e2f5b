// hkv_scheduler.hpp -- step-level scheduler over the paged KV engine and the
// Q4_K backbone (C++ shim, header only; needs the CUDA runtime headers).
#pragma once

#include <array>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "hkv.h"
#include "hkv_pipeline.hpp"

namespace hkv_pipeline {

// One request of the step scheduler: its prompt (text token ids) and how many
// frames of greedy audio codes to generate.  `prefix` optionally names a
// published reference-prompt prefix the request's slot maps copy-on-write.
struct GenerateRequest {
    std::vector<int32_t> prompt_ids;
    int32_t max_frames = 0;
    hkv_prefix_key prefix{};
    bool share_prefix = false;
};

// Step-level scheduler over one engine and its backbone: replaces the
// reference's one-request-at-a-time decode loop (each request runs its own
// per-frame graph through cuda_executor().run_sync, :5133-5177, with audio
// heads micro-batched by AudioHeadBatcher, :3484-3574).  Every step():
//   1. admits queued requests while the slot table and page pool allow
//      (a request that does not fit waits in the queue);
//   2. feeds every request still in its prompt one prompt token, all of them
//      in one hkv_backbone_decode (logits only when one of them finishes its
//      prompt);
//   3. advances every generating request by one frame in one more
//      hkv_backbone_decode: its last codes go up, the new greedy codes come
//      back to the host;
//   4. retires requests with all their frames and releases their slots.
// Requests share the weights read of each projection within a step.  The
// scheduler runs on one host thread; it synchronises `stream` once per step
// (the codes are needed on the host to drive the next step).
class StepScheduler {
  public:
    static constexpr int kCodebooks = 8;
    using Frame = std::array<int32_t, kCodebooks>;

    StepScheduler(PagedKvRuntime &rt, hkv_backbone *bb, int32_t max_batch, hkv_stream stream)
        : rt_(rt), bb_(bb), max_batch_(max_batch), stream_(stream) {
        if (max_batch <= 0) throw std::invalid_argument("StepScheduler: max_batch must be positive");
        hkv_backbone_buffers(bb_, nullptr, nullptr, &dev_codes_out_);
        if (cudaMallocHost(reinterpret_cast<void **>(&host_codes_), sizeof(Frame) * max_batch) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&dev_codes_in_), sizeof(Frame) * max_batch) != cudaSuccess) {
            throw std::runtime_error("StepScheduler: cannot allocate code staging buffers");
        }
    }
    ~StepScheduler() {
        cudaFreeHost(host_codes_);
        cudaFree(dev_codes_in_);
    }
    StepScheduler(const StepScheduler &) = delete;
    StepScheduler &operator=(const StepScheduler &) = delete;

    // Queues a request; returns its id.
    int64_t submit(GenerateRequest req) {
        if (req.prompt_ids.empty() || req.max_frames <= 0) {
            throw std::invalid_argument("StepScheduler: a request needs prompt ids and max_frames > 0");
        }
        const int64_t id = next_id_++;
        queue_.push_back({id, std::move(req)});
        return id;
    }

    // One scheduling step; returns the number of requests still queued or live.
    size_t step() {
        admit();
        std::vector<Live *> prompt, gen;
        for (auto &kv : live_) {
            (kv.second->fed < kv.second->req.prompt_ids.size() ? prompt : gen).push_back(kv.second.get());
        }
        if (!prompt.empty()) run_prompt(prompt);
        if (!gen.empty()) run_generation(gen);
        for (auto it = live_.begin(); it != live_.end();) {
            Live &l = *it->second;
            if (static_cast<int32_t>(l.frames.size()) >= l.req.max_frames) {
                done_[it->first] = std::move(l.frames);
                it = live_.erase(it);  // the slot lease releases the slot
            } else {
                ++it;
            }
        }
        return queue_.size() + live_.size();
    }

    bool finished(int64_t id) const { return done_.count(id) != 0; }
    const std::vector<Frame> &frames(int64_t id) const { return done_.at(id); }
    size_t live() const { return live_.size(); }
    size_t queued() const { return queue_.size(); }

  private:
    struct Live {
        GenerateRequest req;
        ScopedBackendKvCacheSlot slot;
        size_t fed = 0;              // prompt tokens consumed
        bool have_codes = false;     // codes of the last decode are in `last`
        Frame last{};
        std::vector<Frame> frames;
    };

    void admit() {
        while (!queue_.empty() && static_cast<int32_t>(live_.size()) < max_batch_) {
            auto &front = queue_.front();
            const GenerateRequest &r = front.second;
            const int64_t capacity = static_cast<int64_t>(r.prompt_ids.size()) + r.max_frames + 1;
            int32_t slot = -1;
            const int st = hkv_slot_acquire(rt_.engine(), capacity, r.share_prefix ? &r.prefix : nullptr, &slot);
            if (st == HKV_ERR_OOM) {
                break;  // no room yet: retry after requests retire
            }
            check(rt_.engine(), st, "StepScheduler: admit");
            auto l = std::make_unique<Live>();
            l->req = std::move(front.second);
            l->slot = ScopedBackendKvCacheSlot(rt_.engine(), slot);
            l->fed = static_cast<size_t>(l->slot.used());  // a shared prefix is already in the slot
            if (l->fed >= l->req.prompt_ids.size()) {
                // the whole prompt was shared: feed its last token again for the logits
                l->fed = l->req.prompt_ids.size() - 1;
                l->slot.set_used(static_cast<int64_t>(l->fed));
            }
            live_[front.first] = std::move(l);
            queue_.pop_front();
        }
    }

    void read_codes(const std::vector<Live *> &batch) {
        const size_t bytes = sizeof(Frame) * batch.size();
        check(nullptr, cudaMemcpyAsync(host_codes_, dev_codes_out_, bytes, cudaMemcpyDeviceToHost,
                                       static_cast<cudaStream_t>(stream_)) == cudaSuccess ? HKV_OK : HKV_ERR_CUDA,
              "StepScheduler: read codes");
        check(nullptr, cudaStreamSynchronize(static_cast<cudaStream_t>(stream_)) == cudaSuccess ? HKV_OK : HKV_ERR_CUDA,
              "StepScheduler: synchronise");
        check_backbone(hkv_backbone_sync_check(bb_, stream_), "StepScheduler: device check");
        for (size_t e = 0; e < batch.size(); ++e) batch[e]->last = host_codes_[e];
    }

    void run_prompt(const std::vector<Live *> &batch) {
        std::vector<int32_t> ids, slots;
        bool any_last = false;
        for (Live *l : batch) {
            ids.push_back(l->req.prompt_ids[l->fed]);
            slots.push_back(l->slot.slot());
            any_last = any_last || l->fed + 1 == l->req.prompt_ids.size();
        }
        const int32_t n = static_cast<int32_t>(batch.size());
        check_backbone(hkv_backbone_embed_text(bb_, n, ids.data(), stream_), "StepScheduler: embed prompt");
        check_backbone(hkv_backbone_decode(bb_, n, slots.data(), any_last ? 1 : 0, stream_),
                       "StepScheduler: prompt decode");
        for (Live *l : batch) ++l->fed;
        if (any_last) {
            read_codes(batch);
            for (Live *l : batch) {
                if (l->fed == l->req.prompt_ids.size()) l->have_codes = true;
            }
        }
    }

    void run_generation(const std::vector<Live *> &batch) {
        std::vector<Live *> ready;
        for (Live *l : batch) {
            if (l->have_codes) ready.push_back(l);
        }
        if (ready.empty()) return;
        std::vector<int32_t> slots;
        for (size_t e = 0; e < ready.size(); ++e) {
            host_codes_[e] = ready[e]->last;
            slots.push_back(ready[e]->slot.slot());
        }
        const int32_t n = static_cast<int32_t>(ready.size());
        check(nullptr, cudaMemcpyAsync(dev_codes_in_, host_codes_, sizeof(Frame) * ready.size(),
                                       cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream_)) == cudaSuccess
                           ? HKV_OK : HKV_ERR_CUDA,
              "StepScheduler: upload codes");
        check_backbone(hkv_backbone_embed_codes(bb_, n, reinterpret_cast<const int32_t *>(dev_codes_in_), stream_),
                       "StepScheduler: embed codes");
        check_backbone(hkv_backbone_decode(bb_, n, slots.data(), 1, stream_), "StepScheduler: frame decode");
        read_codes(ready);
        for (Live *l : ready) l->frames.push_back(l->last);
    }

    void check_backbone(int status, const char *what) {
        if (status != HKV_OK) {
            throw std::runtime_error(std::string(what) + ": " + hkv_backbone_last_error(bb_));
        }
    }

    PagedKvRuntime &rt_;
    hkv_backbone *bb_;
    int32_t max_batch_;
    hkv_stream stream_;
    int32_t *dev_codes_out_ = nullptr;
    Frame *host_codes_ = nullptr;
    Frame *dev_codes_in_ = nullptr;
    int64_t next_id_ = 0;
    std::deque<std::pair<int64_t, GenerateRequest>> queue_;
    std::map<int64_t, std::unique_ptr<Live>> live_;
    std::map<int64_t, std::vector<Frame>> done_;
};

}  // namespace hkv_pipeline
