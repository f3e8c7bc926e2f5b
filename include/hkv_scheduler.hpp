// hkv_scheduler.hpp -- step-level scheduler over the paged KV engine and the
// Q4_K backbone (C++ shim, header only; needs the CUDA runtime headers).
#pragma once

#include <algorithm>
#include <array>
#include <chrono>
#include <cstdint>
#include <deque>
#include <functional>
#include <limits>
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
    // Cancellation and deadline, as GenerateOptions::cancel / deadline of the
    // reference (throw_if_cancelled, src/higgs_pipeline.cpp:146-153, checked
    // once per frame at :4948): checked between steps; a request whose flag
    // is non-zero, or whose deadline has passed, ends with its frames so far
    // and its slot released.
    const volatile int *cancel = nullptr;
    std::chrono::steady_clock::time_point deadline{};
    // Low-margin window refresh (the reference's fast fallback, :5051-5135,
    // default margin 0.006 at :718-721): when the smallest top-1 / top-2 logit
    // margin over a frame's active codebooks (min(frame + 1, 8), id 1024
    // masked as at :2696-2698) is below refresh_margin, the slot is truncated
    // by the last refresh_window generated rows (0: all of them), those rows
    // are decoded again from their recorded inputs (set_len + re-feed), and the
    // frame's codes are taken from the refreshed logits.  0 turns it off.
    float refresh_margin = 0.f;
    int32_t refresh_window = 0;
};

// How a request ended (or that it has not).
enum class RequestStatus { kQueued, kLive, kDone, kCancelled, kTimedOut };

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
// Before admitting, it ends cancelled and timed-out requests (queued or live)
// between steps, never with a launch of theirs in flight.  Requests share
// the weights read of each projection within a step.  The scheduler runs on
// one host thread; it synchronises `stream` once per step (the codes are
// needed on the host to drive the next step), once more per refreshed
// request.
class StepScheduler {
  public:
    static constexpr int kCodebooks = 8;
    using Frame = std::array<int32_t, kCodebooks>;
    // Host time of step() since the last reset_times(): `wait_us` blocked in
    // the stream synchronisations (the GPU still running the step),
    // `host_us` everything else (planning, launch calls, retirement).
    struct StepTimes {
        int64_t steps = 0;
        double host_us = 0.0;
        double wait_us = 0.0;
    };

    StepScheduler(PagedKvRuntime &rt, hkv_backbone *bb, int32_t max_batch, hkv_stream stream)
        : rt_(rt), bb_(bb), max_batch_(max_batch), stream_(stream) {
        if (max_batch <= 0) throw std::invalid_argument("StepScheduler: max_batch must be positive");
        hkv_backbone_buffers(bb_, nullptr, &dev_logits_, &dev_codes_out_);
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
        const auto t0 = std::chrono::steady_clock::now();
        const double wait0 = times_.wait_us;
        expire();
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
                it = retire(it, RequestStatus::kDone);
            } else {
                ++it;
            }
        }
        const double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
        times_.host_us += us - (times_.wait_us - wait0);
        ++times_.steps;
        return queue_.size() + live_.size();
    }

    // Ended requests: done, cancelled or timed out (frames so far).
    bool finished(int64_t id) const { return done_.count(id) != 0; }
    const std::vector<Frame> &frames(int64_t id) const { return done_.at(id).frames; }
    RequestStatus status(int64_t id) const {
        auto d = done_.find(id);
        if (d != done_.end()) return d->second.status;
        return live_.count(id) != 0 ? RequestStatus::kLive : RequestStatus::kQueued;
    }
    // The reference's exception text for a request that did not finish
    // ("request cancelled", "request timed out"), else empty.
    std::string error(int64_t id) const {
        switch (status(id)) {
            case RequestStatus::kCancelled: return "request cancelled";
            case RequestStatus::kTimedOut: return "request timed out";
            default: return std::string();
        }
    }
    // Window refreshes a request has gone through.
    int32_t refreshes(int64_t id) const {
        auto d = done_.find(id);
        if (d != done_.end()) return d->second.refreshes;
        auto l = live_.find(id);
        return l != live_.end() ? l->second->refreshes : 0;
    }
    const StepTimes &times() const { return times_; }
    void reset_times() { times_ = StepTimes{}; }
    size_t live() const { return live_.size(); }
    size_t queued() const { return queue_.size(); }
    // Prompt steps whose batch held requests at their last prompt token beside
    // requests still inside their prompts.
    int64_t mixed_prompt_steps() const { return mixed_prompt_steps_; }
    // Called with (request id, slot) just before an ended request's slot is
    // released (a test or a cache inspector reads the slot there).
    std::function<void(int64_t, int32_t)> on_retire;

  private:
    struct Live {
        GenerateRequest req;
        ScopedBackendKvCacheSlot slot;
        size_t fed = 0;              // prompt tokens consumed
        bool have_codes = false;     // codes of the last decode are in `last`
        Frame last{};
        std::vector<Frame> frames;
        std::vector<Frame> inputs;   // codes fed by each generation decode
        int32_t refreshes = 0;
    };
    struct Ended {
        RequestStatus status = RequestStatus::kDone;
        std::vector<Frame> frames;
        int32_t refreshes = 0;
    };

    using LiveMap = std::map<int64_t, std::unique_ptr<Live>>;

    LiveMap::iterator retire(LiveMap::iterator it, RequestStatus status) {
        Live &l = *it->second;
        if (on_retire) on_retire(it->first, l.slot.slot());
        Ended &e = done_[it->first];
        e.status = status;
        e.frames = std::move(l.frames);
        e.refreshes = l.refreshes;
        return live_.erase(it);  // the slot lease releases the slot
    }

    static RequestStatus expired(const GenerateRequest &r) {
        if (r.cancel != nullptr && *r.cancel != 0) return RequestStatus::kCancelled;
        if (r.deadline != std::chrono::steady_clock::time_point{} &&
            std::chrono::steady_clock::now() >= r.deadline) {
            return RequestStatus::kTimedOut;
        }
        return RequestStatus::kLive;
    }

    // Ends cancelled and timed-out requests; runs between steps, when no
    // launch of theirs is in flight (each step ends with a synchronisation).
    void expire() {
        for (auto it = queue_.begin(); it != queue_.end();) {
            const RequestStatus st = expired(it->second);
            if (st != RequestStatus::kLive) {
                done_[it->first].status = st;
                it = queue_.erase(it);
            } else {
                ++it;
            }
        }
        for (auto it = live_.begin(); it != live_.end();) {
            const RequestStatus st = expired(it->second->req);
            it = st != RequestStatus::kLive ? retire(it, st) : std::next(it);
        }
    }

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
        synchronise("StepScheduler: synchronise");
        check_backbone(hkv_backbone_sync_check(bb_, stream_), "StepScheduler: device check");
        for (size_t e = 0; e < batch.size(); ++e) batch[e]->last = host_codes_[e];
    }

    void run_prompt(const std::vector<Live *> &batch) {
        std::vector<int32_t> ids, slots;
        bool any_last = false, any_inside = false;
        for (Live *l : batch) {
            ids.push_back(l->req.prompt_ids[l->fed]);
            slots.push_back(l->slot.slot());
            const bool last = l->fed + 1 == l->req.prompt_ids.size();
            any_last = any_last || last;
            any_inside = any_inside || !last;
        }
        if (any_last && any_inside) ++mixed_prompt_steps_;
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

    // Embeds `codes` (host frames) of a batch and decodes it; the codes of
    // the batch are read back when want_logits.
    void decode_codes(const std::vector<Live *> &batch, const std::vector<Frame> &codes,
                      bool want_logits) {
        std::vector<int32_t> slots;
        for (size_t e = 0; e < batch.size(); ++e) {
            host_codes_[e] = codes[e];
            slots.push_back(batch[e]->slot.slot());
        }
        const int32_t n = static_cast<int32_t>(batch.size());
        check(nullptr, cudaMemcpyAsync(dev_codes_in_, host_codes_, sizeof(Frame) * batch.size(),
                                       cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream_)) == cudaSuccess
                           ? HKV_OK : HKV_ERR_CUDA,
              "StepScheduler: upload codes");
        check_backbone(hkv_backbone_embed_codes(bb_, n, reinterpret_cast<const int32_t *>(dev_codes_in_), stream_),
                       "StepScheduler: embed codes");
        check_backbone(hkv_backbone_decode(bb_, n, slots.data(), want_logits ? 1 : 0, stream_),
                       "StepScheduler: frame decode");
        if (want_logits) read_codes(batch);
    }

    // Smallest top-1 / top-2 margin over the active codebooks of entry e's
    // logits (greedy_logits_have_small_margin, :2686-2710; the logits here
    // are codebook-major, [codebook][1026]).
    float min_margin(size_t e, int32_t active) const {
        constexpr int kVocab = 1026, kDataSize = 1024, kEoc = 1025;
        float worst = std::numeric_limits<float>::infinity();
        for (int c = 0; c < std::min(active, kCodebooks); ++c) {
            const float *row = host_logits_.data() + (e * kCodebooks + c) * kVocab;
            float best = -std::numeric_limits<float>::infinity(), second = best;
            for (int v = 0; v < kVocab; ++v) {
                const float x = (v >= kDataSize && v < kEoc) ? -std::numeric_limits<float>::infinity() : row[v];
                if (x > best) {
                    second = best;
                    best = x;
                } else if (x > second) {
                    second = x;
                }
            }
            worst = std::min(worst, best - second);
        }
        return worst;
    }

    // Truncates the last generated rows of `l`'s slot (the window) and
    // decodes them again from their recorded inputs; the last re-decode's
    // codes replace the frame's.
    void refresh(Live *l) {
        const int64_t rows = static_cast<int64_t>(l->inputs.size());
        const int64_t w = l->req.refresh_window > 0 ? std::min<int64_t>(l->req.refresh_window, rows) : rows;
        l->slot.set_used(l->slot.used() - w);
        for (int64_t k = rows - w; k < rows; ++k) {
            decode_codes({l}, {l->inputs[static_cast<size_t>(k)]}, k == rows - 1);
        }
        ++l->refreshes;
    }

    void run_generation(const std::vector<Live *> &batch) {
        std::vector<Live *> ready;
        std::vector<Frame> in;
        bool want_margins = false;
        for (Live *l : batch) {
            if (l->have_codes) {
                ready.push_back(l);
                in.push_back(l->last);
                l->inputs.push_back(l->last);
                want_margins = want_margins || l->req.refresh_margin > 0.f;
            }
        }
        if (ready.empty()) return;
        decode_codes(ready, in, true);
        if (want_margins) {
            host_logits_.resize(ready.size() * kCodebooks * 1026);
            cudaStream_t st = static_cast<cudaStream_t>(stream_);
            check(nullptr, cudaMemcpyAsync(host_logits_.data(), dev_logits_, host_logits_.size() * sizeof(float),
                                           cudaMemcpyDeviceToHost, st) == cudaSuccess ? HKV_OK : HKV_ERR_CUDA,
                  "StepScheduler: read logits");
            synchronise("StepScheduler: synchronise logits");
            std::vector<Live *> low;
            for (size_t e = 0; e < ready.size(); ++e) {
                Live *l = ready[e];
                const int32_t active = std::min<int32_t>(static_cast<int32_t>(l->frames.size()) + 1, kCodebooks);
                if (l->req.refresh_margin > 0.f && min_margin(e, active) < l->req.refresh_margin) {
                    low.push_back(l);
                }
            }
            for (Live *l : low) refresh(l);
        }
        for (Live *l : ready) l->frames.push_back(l->last);
    }

    void synchronise(const char *what) {
        const auto t0 = std::chrono::steady_clock::now();
        const bool ok = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_)) == cudaSuccess;
        times_.wait_us += std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
        check(nullptr, ok ? HKV_OK : HKV_ERR_CUDA, what);
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
    float *dev_logits_ = nullptr;
    Frame *host_codes_ = nullptr;
    Frame *dev_codes_in_ = nullptr;
    std::vector<float> host_logits_;
    int64_t next_id_ = 0;
    int64_t mixed_prompt_steps_ = 0;
    StepTimes times_;
    std::deque<std::pair<int64_t, GenerateRequest>> queue_;
    LiveMap live_;
    std::map<int64_t, Ended> done_;
};

}  // namespace hkv_pipeline
