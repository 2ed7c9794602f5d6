// The training step of apps/train.cpp:212-256 (seampm/tinytrain) as a C ABI,
// for a GPTModel held on the device, plus data parallelism.
//
// Gradients of all parameters live in one flat device arena, laid out in the
// order backward finishes them (final norm, last block ... first block, the
// tied embedding last). With a communicator, the arena is cut into buckets of
// about bucket_bytes; during the last micro-batch's backward the autograd
// engine reports each parameter whose gradient is final, and a bucket whose
// parameters are all final is all-reduced on a separate comm stream while
// backward continues. The compute stream waits for the last bucket before
// the fused clip + AdamW kernel, which divides by world * n_micro.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <functional>
#include <thread>
#include <chrono>
#include <unistd.h>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>

#include "internal.h"
#include "tinytrain/model.h"
#include "tinytrain/optim.h"
#include "tt_trainer.h"
#include "ttk.h"

extern "C" int64_t ttk_launch_count(void);

namespace {

thread_local std::string t_err;

using namespace tt;
using namespace tt::detail;

struct Bucket {
    int64_t offset = 0, count = 0;  // elements in the arena
    int pending = 0;                // parameters not yet final this step
    int total = 0;
};

// Arena layout and bucket plan for parameters of the given sizes (in
// parameters() order): parameter i gets arena offset offs[i]; parameters are
// placed in reverse order (the order backward finishes them) on 64-element
// (256-byte) boundaries; consecutive parameters are grouped into buckets of
// at most cap elements (a larger parameter gets a bucket of its own).
int64_t plan_arena(const std::vector<int64_t>& sizes, int64_t cap, std::vector<int64_t>& offs,
                   std::vector<Bucket>& buckets, std::vector<int>& bucket_of_param) {
    const size_t n = sizes.size();
    offs.assign(n, 0);
    bucket_of_param.assign(n, 0);
    buckets.clear();
    int64_t off = 0;
    Bucket cur;
    for (size_t k = n; k-- > 0;) {
        const int64_t span = (sizes[k] + 63) / 64 * 64;
        offs[k] = off;
        if (cur.total > 0 && cur.count + span > cap) {
            buckets.push_back(cur);
            cur = Bucket();
            cur.offset = off;
        }
        cur.count += span;
        cur.total += 1;
        bucket_of_param[k] = static_cast<int>(buckets.size());
        off += span;
    }
    if (cur.total > 0)
        buckets.push_back(cur);
    return off;
}

// Bounded wait for the collectives of a data-parallel step (the reference has
// no distributed code; this is the failure path of the exchange step). Polls
// `done` every poll_ms and, while waiting, `async_error` (the communicator's
// asynchronous error state). On an error, or once timeout_s has passed (a
// peer that left or hangs never joins the collective), calls `abort` once and
// returns 1 (error) or 2 (timeout) with the reason in `why`; 0 when done.
int watch_collectives(const std::function<int()>& done, const std::function<int()>& async_error,
                      const std::function<void()>& abort, double timeout_s, double poll_ms,
                      std::string& why) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        if (done())
            return 0;
        if (async_error()) {
            why = "the communicator reported an asynchronous error; aborted";
            abort();
            return 1;
        }
        const double waited =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (waited > timeout_s) {
            why = "collectives did not complete within " + std::to_string(timeout_s) +
                  " s (a peer left or hangs); aborted";
            abort();
            return 2;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(static_cast<int64_t>(poll_ms * 1e3)));
    }
}

struct Trainer {
    GPTConfig cfg;
    std::unique_ptr<GPTModel> model;
    std::vector<Tensor*> params;
    std::unique_ptr<AdamW> opt;
    tt_adamw_config ocfg{3e-4f, 0.9f, 0.95f, 1e-8f, 0.1f, 1.0f};
    float* arena = nullptr;
    int64_t arena_n = 0;
    std::vector<int64_t> param_offset;  // arena offset per parameter
    float* loss_acc = nullptr;          // device: sum of micro-batch losses
    float* loss_out = nullptr;          // device: step loss
    // data parallelism
    void* comm = nullptr;
    int rank = 0, world = 1;
    void* comm_stream = nullptr;
    std::vector<Bucket> buckets;
    std::unordered_map<Tensor::Impl*, int> bucket_of;
    std::vector<void*> bucket_events;
    void* done_event = nullptr;
    // collective watchdog: the ends of the distributed steps in flight (at
    // most two: the host enqueues a step while the previous one runs)
    std::vector<void*> step_events;  // oldest first
    std::vector<void*> spare_events;
    double coll_timeout_s = 300.0;
    std::string dist_error;  // set once the communicator was aborted
    // Optional timing of the gradient all-reduce: per bucket, events around
    // its all-reduce on the comm stream; per step, the compute stream's end
    // of backward against the end of the last all-reduce (the exposed tail).
    bool comm_prof = false;
    struct CommRec {
        void *a, *b;
    };
    std::vector<CommRec> comm_recs, tail_recs;
    std::vector<void*> event_pool;
    void* pooled_event() {
        void* e = nullptr;
        if (!event_pool.empty()) {
            e = event_pool.back();
            event_pool.pop_back();
        } else {
            check(ttk_event_create(&e), "event");
        }
        return e;
    }

    ~Trainer() {
        tt::set_grad_ready_hook(nullptr);
        try {
            wait_dist();
        } catch (const std::exception&) {
        }
        void* s = stream_if_ready();
        if (s)
            ttk_stream_synchronize(s);
        if (comm)
            ttk_dist_destroy(comm);
        for (void* e : step_events)
            ttk_event_destroy(e);
        for (void* e : spare_events)
            ttk_event_destroy(e);
        for (auto& sl : async_slots) {
            ttk_host_free(sl.ids);
            ttk_host_free(sl.out);
            ttk_free(sl.dev, s);
            if (sl.done)
                ttk_event_destroy(sl.done);
        }
        for (auto& r : comm_recs)
            event_pool.push_back(r.a), event_pool.push_back(r.b);
        for (auto& r : tail_recs)
            event_pool.push_back(r.a), event_pool.push_back(r.b);
        for (void* e : event_pool)
            ttk_event_destroy(e);
        for (void* e : bucket_events)
            ttk_event_destroy(e);
        if (done_event)
            ttk_event_destroy(done_event);
        ttk_graph_destroy(graph_exec);
        if (capture_stream)
            ttk_stream_destroy(capture_stream);
        ttk_free(sched, s);
        if (comm_stream)
            ttk_stream_destroy(comm_stream);
        opt.reset();
        model.reset();
        ttk_free(arena, s);
        ttk_free(loss_acc, s);
        ttk_free(loss_out, s);
    }

    void setup() {
        params = model->parameters();
        std::vector<int64_t> sizes;
        for (Tensor* p : params)
            sizes.push_back(p->numel());
        std::vector<Bucket> unused;
        std::vector<int> unused_ids;
        arena_n = plan_arena(sizes, INT64_MAX, param_offset, unused, unused_ids);
        check(ttk_malloc(reinterpret_cast<void**>(&arena), static_cast<size_t>(arena_n) * 4,
                         stream()),
              "grad arena");
        check(ttk_memset(arena, 0, static_cast<size_t>(arena_n) * 4, stream()), "grad arena");
        for (size_t i = 0; i < params.size(); ++i) {
            auto buf = std::make_shared<Buffer>(params[i]->numel());
            buf->dev = arena + param_offset[i];
            buf->external = true;
            buf->fill(0.0f);
            params[i]->impl()->grad = buf;
        }
        check(ttk_malloc(reinterpret_cast<void**>(&loss_acc), 16, stream()), "loss");
        check(ttk_malloc(reinterpret_cast<void**>(&loss_out), 16, stream()), "loss");
        opt.reset(new AdamW(params, ocfg.lr, ocfg.beta1, ocfg.beta2, ocfg.eps, ocfg.weight_decay));
        opt->set_clip_norm(ocfg.clip_norm);
    }

    void zero_grads() {
        // One memset of the arena; each parameter's gradient is then "fresh"
        // (logically zero) so its first contribution overwrites.
        for (Tensor* p : params)
            p->impl()->grad->fill(0.0f);
    }

    void make_buckets(int64_t bucket_bytes) {
        const int64_t cap = std::max<int64_t>(bucket_bytes / 4, 1 << 16);
        std::vector<int64_t> sizes;
        for (Tensor* p : params)
            sizes.push_back(p->numel());
        std::vector<int> ids;
        plan_arena(sizes, cap, param_offset, buckets, ids);
        bucket_of.clear();
        for (size_t i = 0; i < params.size(); ++i)
            bucket_of[params[i]->impl().get()] = ids[i];
        for (void* e : bucket_events)
            ttk_event_destroy(e);
        bucket_events.assign(buckets.size(), nullptr);
        for (auto& e : bucket_events)
            check(ttk_event_create(&e), "event");
        if (!done_event)
            check(ttk_event_create(&done_event), "event");
    }

    void launch_bucket(int b) {
        Bucket& bk = buckets[static_cast<size_t>(b)];
        check(ttk_event_record(bucket_events[static_cast<size_t>(b)], stream()), "record");
        check(ttk_stream_wait_event(comm_stream, bucket_events[static_cast<size_t>(b)]), "wait");
        CommRec r{nullptr, nullptr};
        if (comm_prof) {
            r = {pooled_event(), pooled_event()};
            check(ttk_event_record(r.a, comm_stream), "record");
        }
        check(ttk_dist_allreduce_f32(comm, arena + bk.offset, bk.count, comm_stream), "allreduce");
        if (comm_prof) {
            check(ttk_event_record(r.b, comm_stream), "record");
            comm_recs.push_back(r);
        }
    }

    // TT_TRACE_STEP=1: host-side timestamps of each micro-batch's enqueue
    // (start of forward, end of backward) on stderr, to tell host stalls
    // from device time.
    bool trace = [] {
        const char* e = std::getenv("TT_TRACE_STEP");
        return e && e[0] == '1';
    }();
    std::chrono::steady_clock::time_point trace_t0;
    void trace_mark(const char* what, int64_t m) {
        if (!trace)
            return;
        const auto now = std::chrono::steady_clock::now();
        const double ms = std::chrono::duration<double, std::milli>(now - trace_t0).count();
        const double abs_ms =
            std::chrono::duration<double, std::milli>(now.time_since_epoch()).count();
        std::fprintf(stderr, "tt_trace %d %s %ld %.2f %.2f\n", static_cast<int>(getpid()), what,
                     static_cast<long>(m), ms, abs_ms);
    }

    // Runs fwd+bwd over n_micro micro-batches; ids are device pointers.
    void accumulate(const int64_t* idx, const int64_t* tgt, int64_t B, int64_t T,
                    int64_t n_micro) {
        check(ttk_memset(loss_acc, 0, 4, stream()), "loss zero");
        const int64_t per = B * T;
        for (int64_t m = 0; m < n_micro; ++m) {
            trace_mark("fwd", m);
            const bool last = m + 1 == n_micro;
            if (comm && last) {
                for (auto& bk : buckets)
                    bk.pending = bk.total;
                tt::set_grad_ready_hook([this](const std::shared_ptr<Tensor::Impl>& p) {
                    auto it = bucket_of.find(p.get());
                    if (it == bucket_of.end())
                        return;
                    if (--buckets[static_cast<size_t>(it->second)].pending == 0)
                        launch_bucket(it->second);
                });
            }
            {
                Tensor logits = model->forward(DeviceIds::borrow(idx + m * per, per), B, T);
                Tensor loss = cross_entropy(logits, DeviceIds::borrow(tgt + m * per, per));
                check(ttk_axpy(1.0f, loss.device_data(), loss_acc, 1, stream()), "loss acc");
                trace_mark("bwd", m);
                loss.backward();
            }
            trace_mark("done", m);
            if (comm && last) {
                tt::set_grad_ready_hook(nullptr);
                // Any bucket whose parameters got no gradient this step.
                for (size_t b = 0; b < buckets.size(); ++b)
                    if (buckets[b].pending > 0)
                        launch_bucket(static_cast<int>(b));
                check(ttk_event_record(done_event, comm_stream), "record");
                if (comm_prof) {
                    CommRec r{pooled_event(), pooled_event()};
                    check(ttk_event_record(r.a, stream()), "record");  // backward done
                    check(ttk_event_record(r.b, comm_stream), "record");  // all-reduces done
                    tail_recs.push_back(r);
                }
                check(ttk_stream_wait_event(stream(), done_event), "wait");
            }
        }
        // Step loss = mean over micro-batches (and ranks).
        check(ttk_fill(loss_out, 0.0f, 1, stream()), "loss");
        check(ttk_axpy(1.0f / static_cast<float>(n_micro), loss_acc, loss_out, 1, stream()), "loss");
        if (comm) {
            check(ttk_dist_allreduce_f32(comm, loss_out, 1, stream()), "loss allreduce");
            const float inv = 1.0f / static_cast<float>(world);
            check(ttk_fill(loss_acc, 0.0f, 1, stream()), "loss");
            check(ttk_axpy(inv, loss_out, loss_acc, 1, stream()), "loss");
            check(ttk_memcpy_d2d(loss_out, loss_acc, 4, stream()), "loss");
        }
    }

    void optimizer_step(int64_t n_micro, float lr) {
        opt->set_lr(lr);
        opt->set_grad_scale(1.0f / static_cast<float>(n_micro * world));
        opt->step();
    }

    // Distributed steps: before a step, at most one earlier step may still be
    // running (the host enqueues a step while the previous one executes); an
    // older one must have completed within the deadline. After a step its
    // end is recorded for these checks.
    void begin_step() {
        if (!dist_error.empty())
            throw std::runtime_error("data-parallel step refused: the communicator was aborted (" +
                                     dist_error + ")");
        while (step_events.size() >= 2)
            wait_oldest();
    }

    void end_step() {
        if (!comm)
            return;
        void* e = nullptr;
        if (!spare_events.empty()) {
            e = spare_events.back();
            spare_events.pop_back();
        } else {
            check(ttk_event_create(&e), "event");
        }
        check(ttk_event_record(e, stream()), "record");
        step_events.push_back(e);
    }

    // Every recorded step end, each with the bounded wait.
    void wait_dist() {
        while (comm && !step_events.empty())
            wait_oldest();
    }

    // Bounded wait for the oldest recorded step end. On an asynchronous NCCL
    // error or a deadline overrun (a peer left or hangs) the communicator is
    // aborted, which ends the pending collectives, and the step throws.
    void wait_oldest() {
        if (!comm || step_events.empty())
            return;
        void* ev = step_events.front();
        std::string why;
        const int rc = watch_collectives(
            [&] {
                int d = 0;
                check(ttk_event_query(ev, &d), "event query");
                return d;
            },
            [&] {
                int e = 0;
                return ttk_dist_async_error(comm, &e) != TTK_OK || e != 0 ? 1 : 0;
            },
            [&] { ttk_dist_abort(comm); }, coll_timeout_s, 1.0, why);
        step_events.erase(step_events.begin());
        spare_events.push_back(ev);
        if (rc == 0)
            return;
        comm = nullptr;  // freed by the abort
        dist_error = why;
        for (void* e : step_events)
            spare_events.push_back(e);
        step_events.clear();
        ttk_stream_synchronize(stream());  // the aborted collectives have returned
        if (comm_stream)
            ttk_stream_synchronize(comm_stream);
        throw std::runtime_error("data-parallel step: " + why);
    }

    // Pipelined steps (tt_trainer_step_submit / tt_trainer_step_result): two
    // slots, each with pinned staging for the ids, device ids, pinned space
    // for the loss and the squared gradient norm, and a completion event.
    struct AsyncSlot {
        int64_t* ids = nullptr;  // pinned: idx then targets
        int64_t* dev = nullptr;
        size_t cap = 0;          // ids per slot (idx + targets)
        double* out = nullptr;   // pinned: [0] loss (as float bits), [1] sum of squares
        void* done = nullptr;
        bool pending = false;
        float scale = 1.0f;      // gradient scale of the step (for the norm)
        bool has_norm = false;
    };
    AsyncSlot async_slots[2];
    int async_next = 0, async_oldest = 0;

    // Steps replayed from a CUDA graph (tt_trainer_step_graph). The graph
    // holds one recorded step for fixed id pointers and sizes; the AdamW
    // kernel in it reads {lr, lr_t} from `sched`, written before each launch.
    struct GraphKey {
        const int64_t* idx = nullptr;
        const int64_t* tgt = nullptr;
        int64_t B = 0, T = 0, n_micro = 0;
        bool operator==(const GraphKey& o) const {
            return idx == o.idx && tgt == o.tgt && B == o.B && T == o.T && n_micro == o.n_micro;
        }
    };
    GraphKey graph_key, warm_key;
    bool warm_valid = false;
    void* graph_exec = nullptr;
    void* capture_stream = nullptr;
    float* sched = nullptr;

    // Drops the recorded step: anything that replaces or rewrites the state
    // a graph reads (parameters written from the host, a new optimizer,
    // loaded checkpoints, a communicator) calls this, so the next
    // tt_trainer_step_graph runs eagerly (uploading host-side writes) and
    // records again.
    void drop_graph() {
        if (graph_exec) {
            check(ttk_stream_synchronize(stream()), "graph release");
            ttk_graph_destroy(graph_exec);
            graph_exec = nullptr;
        }
        warm_valid = false;
    }

    // Records one training step on the capture stream (nothing runs while
    // recording; the host-side state advances by one step, as for an eager
    // step) and instantiates it. The pool's unused memory is returned to the
    // device first: the graph allocates its activations from its own pool.
    void capture_step(const GraphKey& key, float lr) {
        if (!capture_stream)
            check(ttk_stream_create(&capture_stream), "capture stream");
        if (!sched)
            check(ttk_malloc(reinterpret_cast<void**>(&sched), 16, stream()), "schedule");
        void* user = stream();
        check(ttk_pool_trim(user), "pool trim");
        tt::set_stream(capture_stream);
        opt->set_device_schedule(sched);
        const int64_t step0 = opt->step_count();
        std::exception_ptr err;
        int rc = ttk_stream_begin_capture(capture_stream);
        if (!rc) {
            try {
                begin_step();
                zero_grads();
                accumulate(key.idx, key.tgt, key.B, key.T, key.n_micro);
                optimizer_step(key.n_micro, lr);
                end_step();
            } catch (...) {
                err = std::current_exception();
            }
            void* exec = nullptr;
            const int rc_end = ttk_stream_end_capture(capture_stream, &exec);
            if (!rc_end && !err) {
                graph_exec = exec;
                graph_key = key;
            } else {
                ttk_graph_destroy(exec);
                rc = rc_end;
            }
        }
        const std::string msg = rc ? ttk_last_error() : "";
        opt->set_device_schedule(nullptr);
        tt::set_stream(user);
        if (err || rc) {
            // nothing ran: the step count stays; the next call runs eagerly
            opt->set_step_count(step0);
            warm_valid = false;
        }
        if (err)
            std::rethrow_exception(err);
        if (rc)
            throw std::runtime_error("step_graph: capture failed: " + msg);
    }
};

// A token stream resident in device memory (int32, apps/prepare_data.cpp's
// file format), plus a pinned staging buffer for window starts.
struct Tokens {
    int32_t* dev = nullptr;
    int64_t n = 0;
    ~Tokens() { ttk_free(dev, stream_if_ready()); }
};

Tokens* make_tokens(const int32_t* host, int64_t n) {
    if (n < 2)
        throw std::invalid_argument("tokens: need at least 2 tokens");
    ensure_runtime();
    auto t = std::make_unique<Tokens>();
    t->n = n;
    check(ttk_malloc(reinterpret_cast<void**>(&t->dev), static_cast<size_t>(n) * 4, stream()),
          "tokens");
    check(ttk_memcpy_h2d(t->dev, host, static_cast<size_t>(n) * 4, stream()), "tokens upload");
    check(ttk_stream_synchronize(stream()), "tokens upload");
    return t.release();
}

uint64_t xorshift_next(uint64_t& s) {  // apps/train.cpp:145-153
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1DULL;
}

// safetensors writer / reader for flat float32 tensors (the format of
// model.safetensors: 8-byte header length, JSON header, payloads).
void write_safetensors(const std::string& path,
                       const std::vector<std::pair<std::string, std::pair<int64_t, const float*>>>&
                           tensors,
                       const std::string& metadata_json) {
    std::map<std::string, std::string> entries;
    int64_t off = 0;
    for (auto& [name, t] : tensors) {
        entries[name] = "{\"data_offsets\":[" + std::to_string(off) + "," +
                        std::to_string(off + t.first * 4) + "],\"dtype\":\"F32\",\"shape\":[" +
                        std::to_string(t.first) + "]}";
        off += t.first * 4;
    }
    std::string header = "{\"__metadata__\":" + metadata_json;
    for (auto& [k, v] : entries)
        header += ",\"" + k + "\":" + v;
    header += "}";
    std::ofstream f(path, std::ios::binary);
    if (!f)
        throw std::runtime_error("save: cannot open " + path);
    const uint64_t hlen = header.size();
    f.write(reinterpret_cast<const char*>(&hlen), 8);
    f.write(header.data(), static_cast<std::streamsize>(header.size()));
    for (auto& [name, t] : tensors)
        f.write(reinterpret_cast<const char*>(t.second), static_cast<std::streamsize>(t.first * 4));
    if (!f)
        throw std::runtime_error("save: write failed for " + path);
}

// Reads the header of a safetensors file; returns it and the payload start.
std::string read_header(std::ifstream& f, const std::string& path) {
    uint64_t hlen = 0;
    f.read(reinterpret_cast<char*>(&hlen), 8);
    if (!f || hlen > (1ull << 30))
        throw std::runtime_error("load: bad header in " + path);
    std::string h(static_cast<size_t>(hlen), '\0');
    f.read(h.data(), static_cast<std::streamsize>(hlen));
    return h;
}

// Offsets of tensor `name` in a header written by write_safetensors.
bool find_tensor(const std::string& h, const std::string& name, uint64_t& beg, uint64_t& end) {
    const size_t at = h.find("\"" + name + "\":{");
    if (at == std::string::npos)
        return false;
    const size_t p = h.find("\"data_offsets\":[", at);
    return p != std::string::npos &&
           std::sscanf(h.c_str() + p, "\"data_offsets\":[%lu,%lu]", &beg, &end) == 2;
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        t_err = e.what();
        return 1;
    }
}

Trainer* T_(void* h) { return static_cast<Trainer*>(h); }

}  // namespace

extern "C" {

const char* tt_last_error(void) { return t_err.c_str(); }

int64_t tt_kernel_launches(void) { return ttk_launch_count(); }
int64_t tt_fused_attention_chains(void) { return tt::fused_attention_chains(); }

int tt_trainer_create(const tt_model_config* c, uint64_t seed, int host_init, void** handle) {
    return guarded([&] {
        auto tr = std::make_unique<Trainer>();
        tr->cfg.vocab_size = c->vocab;
        tr->cfg.dim = c->dim;
        tr->cfg.n_layers = c->layers;
        tr->cfg.n_heads = c->heads;
        tr->cfg.n_kv_heads = c->heads;
        tr->cfg.ffn_dim = c->ffn;
        tr->cfg.max_seq_len = c->max_seq;
        tr->cfg.norm_eps = c->norm_eps;
        tr->cfg.rope_theta = c->rope_theta;
        tr->model.reset(new GPTModel(tr->cfg, seed, host_init != 0));
        tr->setup();
        *handle = tr.release();
    });
}

int tt_trainer_destroy(void* h) {
    return guarded([&] { delete T_(h); });
}

int tt_trainer_set_stream(void* h, void* s) {
    // The stream is process-wide; h may be NULL (call before creating).
    return guarded([&] {
        (void)h;
        tt::set_stream(s);
    });
}

int64_t tt_trainer_param_count(void* h) {
    int64_t n = 0;
    for (Tensor* p : T_(h)->params)
        n += p->numel();
    return n;
}

int tt_trainer_init_normal(void* h, float std, uint64_t seed) {
    return guarded([&] {
        T_(h)->drop_graph();
        T_(h)->model->init_normal_(std, seed);
    });
}

int tt_trainer_set_params(void* h, const float* host, int64_t n) {
    return guarded([&] {
        if (n != tt_trainer_param_count(h))
            throw std::invalid_argument("set_params: size mismatch");
        T_(h)->drop_graph();
        int64_t off = 0;
        for (Tensor* p : T_(h)->params) {
            p->copy_from_host(host + off);
            off += p->numel();
        }
    });
}

int tt_trainer_get_params(void* h, float* host, int64_t n) {
    return guarded([&] {
        if (n != tt_trainer_param_count(h))
            throw std::invalid_argument("get_params: size mismatch");
        int64_t off = 0;
        for (Tensor* p : T_(h)->params) {
            p->copy_to_host(host + off);
            off += p->numel();
        }
    });
}

int tt_trainer_get_grads(void* h, float* host, int64_t n) {
    return guarded([&] {
        if (n != tt_trainer_param_count(h))
            throw std::invalid_argument("get_grads: size mismatch");
        int64_t off = 0;
        for (Tensor* p : T_(h)->params) {
            const float* g = p->grad_data();
            std::memcpy(host + off, g, static_cast<size_t>(p->numel()) * 4);
            off += p->numel();
        }
    });
}

int tt_trainer_set_optimizer(void* h, const tt_adamw_config* c) {
    return guarded([&] {
        Trainer* t = T_(h);
        t->drop_graph();
        t->ocfg = *c;
        t->opt.reset(new AdamW(t->params, c->lr, c->beta1, c->beta2, c->eps, c->weight_decay));
        t->opt->set_clip_norm(c->clip_norm);
    });
}

int tt_trainer_step_device(void* h, const int64_t* idx, const int64_t* targets, int64_t B,
                           int64_t T, int64_t n_micro, float lr) {
    return guarded([&] {
        Trainer* t = T_(h);
        if (B <= 0 || T <= 0 || n_micro <= 0)
            throw std::invalid_argument("step: sizes must be positive");
        t->trace_t0 = std::chrono::steady_clock::now();
        t->trace_mark("step", 0);
        t->begin_step();
        t->zero_grads();
        t->accumulate(idx, targets, B, T, n_micro);
        t->optimizer_step(n_micro, lr);
        t->end_step();
        t->trace_mark("enqueued", 0);
    });
}

int tt_trainer_step_graph(void* h, const int64_t* idx, const int64_t* targets, int64_t B,
                          int64_t T, int64_t n_micro, float lr) {
    return guarded([&] {
        Trainer* t = T_(h);
        if (B <= 0 || T <= 0 || n_micro <= 0 || !idx || !targets)
            throw std::invalid_argument("step: sizes must be positive");
        if (t->comm)
            throw std::logic_error(
                "step_graph: data-parallel steps are not recorded in a graph; use step_device");
        const Trainer::GraphKey key{idx, targets, B, T, n_micro};
        if (t->graph_exec && !(t->graph_key == key))
            t->drop_graph();
        if (!t->graph_exec) {
            if (!t->warm_valid || !(t->warm_key == key)) {
                // The first step with these ids and sizes runs eagerly: it
                // allocates the state (moments, cached weight splits) that
                // the recorded step then finds in place.
                t->begin_step();
                t->zero_grads();
                t->accumulate(idx, targets, B, T, n_micro);
                t->optimizer_step(n_micro, lr);
                t->end_step();
                t->warm_key = key;
                t->warm_valid = true;
                return;
            }
            t->capture_step(key, lr);  // the optimizer's step count advanced by one
        } else {
            t->opt->set_step_count(t->opt->step_count() + 1);
        }
        check(ttk_adamw_sched_set(t->sched, lr, t->ocfg.beta1, t->ocfg.beta2,
                                  t->opt->step_count(), stream()),
              "schedule");
        check(ttk_graph_launch(t->graph_exec, stream()), "graph launch");
    });
}

int tt_trainer_step(void* h, const int64_t* idx, const int64_t* targets, int64_t B, int64_t T,
                    int64_t n_micro, float lr, float* loss, float* grad_norm) {
    return guarded([&] {
        Trainer* t = T_(h);
        t->trace_t0 = std::chrono::steady_clock::now();
        t->trace_mark("step", 0);
        const int64_t n = B * T * n_micro;
        if (B <= 0 || T <= 0 || n_micro <= 0)
            throw std::invalid_argument("step: sizes must be positive");
        for (int64_t i = 0; i < n; ++i)
            if (idx[i] < 0 || idx[i] >= t->cfg.vocab_size || targets[i] < 0 ||
                targets[i] >= t->cfg.vocab_size)
                throw std::invalid_argument("embedding: index out of range");
        Scratch d(static_cast<size_t>(n) * 16);
        check(ttk_memcpy_h2d(d.ptr, idx, static_cast<size_t>(n) * 8, stream()), "ids");
        check(ttk_memcpy_h2d(d.as<int64_t>() + n, targets, static_cast<size_t>(n) * 8, stream()),
              "ids");
        t->begin_step();
        t->zero_grads();
        t->accumulate(d.as<int64_t>(), d.as<int64_t>() + n, B, T, n_micro);
        t->optimizer_step(n_micro, lr);
        t->end_step();
        t->wait_dist();  // bounded, before the blocking loss read
        t->trace_mark("enqueued", 0);
        if (loss)
            check(ttk_memcpy_d2h(loss, t->loss_out, 4, stream()), "loss read");
        t->trace_mark("loss", 0);
        if (grad_norm)
            *grad_norm = t->ocfg.clip_norm > 0.0f ? t->opt->last_grad_norm() : 0.0f;
    });
}

int tt_trainer_step_submit(void* h, const int64_t* idx, const int64_t* targets, int64_t B,
                           int64_t T, int64_t n_micro, float lr) {
    return guarded([&] {
        Trainer* t = T_(h);
        const int64_t n = B * T * n_micro;
        if (B <= 0 || T <= 0 || n_micro <= 0)
            throw std::invalid_argument("step: sizes must be positive");
        Trainer::AsyncSlot& sl = t->async_slots[t->async_next];
        if (sl.pending)
            throw std::logic_error(
                "step_submit: two steps are in flight; collect the oldest with step_result first");
        for (int64_t i = 0; i < n; ++i)
            if (idx[i] < 0 || idx[i] >= t->cfg.vocab_size || targets[i] < 0 ||
                targets[i] >= t->cfg.vocab_size)
                throw std::invalid_argument("embedding: index out of range");
        if (sl.cap < static_cast<size_t>(2 * n)) {
            if (sl.done)
                check(ttk_event_synchronize(sl.done), "slot reuse");  // no copy still reads it
            ttk_host_free(sl.ids);
            ttk_free(sl.dev, stream());
            sl.ids = nullptr;
            sl.dev = nullptr;
            check(ttk_host_alloc(reinterpret_cast<void**>(&sl.ids), static_cast<size_t>(n) * 16),
                  "pinned ids");
            check(ttk_malloc(reinterpret_cast<void**>(&sl.dev), static_cast<size_t>(n) * 16,
                             stream()),
                  "device ids");
            sl.cap = static_cast<size_t>(2 * n);
        }
        if (!sl.out)
            check(ttk_host_alloc(reinterpret_cast<void**>(&sl.out), 16), "pinned result");
        if (!sl.done)
            check(ttk_event_create(&sl.done), "event");
        // The slot's previous upload finished before its result was collected,
        // so the staging memory is free.
        std::memcpy(sl.ids, idx, static_cast<size_t>(n) * 8);
        std::memcpy(sl.ids + n, targets, static_cast<size_t>(n) * 8);
        check(ttk_memcpy_h2d(sl.dev, sl.ids, static_cast<size_t>(n) * 16, stream()), "ids");
        t->begin_step();
        t->zero_grads();
        t->accumulate(sl.dev, sl.dev + n, B, T, n_micro);
        t->optimizer_step(n_micro, lr);
        t->end_step();
        check(ttk_memcpy_d2h_async(sl.out, t->loss_out, 4, stream()), "loss read");
        const double* ss = t->opt->grad_sumsq_device();
        sl.has_norm = t->ocfg.clip_norm > 0.0f && ss;
        sl.scale = t->opt->grad_scale();
        if (sl.has_norm)
            check(ttk_memcpy_d2h_async(sl.out + 1, ss, 8, stream()), "norm read");
        check(ttk_event_record(sl.done, stream()), "record");
        sl.pending = true;
        t->async_next ^= 1;
    });
}

int tt_trainer_step_result(void* h, float* loss, float* grad_norm) {
    return guarded([&] {
        Trainer* t = T_(h);
        Trainer::AsyncSlot& sl = t->async_slots[t->async_oldest];
        if (!sl.pending)
            throw std::logic_error("step_result: no step in flight");
        t->wait_dist();  // bounded wait on the collectives (distributed runs)
        check(ttk_event_synchronize(sl.done), "step result");
        sl.pending = false;
        t->async_oldest ^= 1;
        if (loss)
            std::memcpy(loss, sl.out, 4);
        if (grad_norm)
            *grad_norm = sl.has_norm ? static_cast<float>(std::sqrt(sl.out[1]) * sl.scale) : 0.0f;
    });
}

int tt_trainer_last_loss(void* h, float* loss) {
    return guarded([&] { check(ttk_memcpy_d2h(loss, T_(h)->loss_out, 4, stream()), "loss read"); });
}

int tt_trainer_forward_backward(void* h, const int64_t* idx, const int64_t* targets, int64_t B,
                                int64_t T, float* loss, float* logits) {
    return guarded([&] {
        Trainer* t = T_(h);
        std::vector<int64_t> ix(idx, idx + B * T), tg(targets, targets + B * T);
        t->zero_grads();
        Tensor lg = t->model->forward(ix, B, T);
        if (logits)
            lg.copy_to_host(logits);
        Tensor l = cross_entropy(lg, tg);
        if (loss)
            l.copy_to_host(loss);
        l.backward();
        tt::synchronize();
    });
}

int tt_tokens_from_host(const int32_t* host, int64_t n, void** tokens) {
    return guarded([&] {
        if (!host || !tokens)
            throw std::invalid_argument("tokens: null pointer");
        *tokens = make_tokens(host, n);
    });
}

int tt_tokens_from_file(const char* path, void** tokens) {
    return guarded([&] {
        std::ifstream f(path, std::ios::binary | std::ios::ate);
        if (!f)
            throw std::runtime_error(std::string("tokens: cannot open ") + path);
        const int64_t nbytes = f.tellg();
        f.seekg(0);
        std::vector<int32_t> tok(static_cast<size_t>(nbytes / 4));
        f.read(reinterpret_cast<char*>(tok.data()), static_cast<std::streamsize>(tok.size() * 4));
        if (!f)
            throw std::runtime_error(std::string("tokens: read failed for ") + path);
        *tokens = make_tokens(tok.data(), static_cast<int64_t>(tok.size()));
    });
}

int64_t tt_tokens_count(void* tokens) { return tokens ? static_cast<Tokens*>(tokens)->n : 0; }

int tt_tokens_destroy(void* tokens) {
    return guarded([&] { delete static_cast<Tokens*>(tokens); });
}

int tt_sample_windows(uint64_t* rng_state, int64_t ntok, int64_t T, int64_t count,
                      int64_t* starts) {
    return guarded([&] {
        if (!rng_state || (count > 0 && !starts) || T <= 0 || ntok - T - 1 <= 0)
            throw std::invalid_argument("sample_windows: need ntok > T + 1");
        uint64_t s = *rng_state ? *rng_state : 0x9E3779B97F4A7C15ULL;
        const uint64_t range = static_cast<uint64_t>(ntok - T - 1);
        for (int64_t i = 0; i < count; ++i)
            starts[i] = static_cast<int64_t>(xorshift_next(s) % range);
        *rng_state = s;
    });
}

int tt_trainer_step_tokens(void* h, void* tokens, const int64_t* starts, int64_t B, int64_t T,
                           int64_t n_micro, float lr, float* loss, float* grad_norm) {
    return guarded([&] {
        Trainer* t = T_(h);
        Tokens* tk = static_cast<Tokens*>(tokens);
        if (!tk || !starts || B <= 0 || T <= 0 || n_micro <= 0)
            throw std::invalid_argument("step_tokens: bad arguments");
        const int64_t w = B * n_micro;
        for (int64_t i = 0; i < w; ++i)
            if (starts[i] < 0 || starts[i] + T >= tk->n)
                throw std::invalid_argument("step_tokens: window out of range");
        // ids and targets for every micro-batch, then the window starts
        Scratch d(static_cast<size_t>(w * T) * 16 + static_cast<size_t>(w) * 8);
        int64_t* idx = d.as<int64_t>();
        int64_t* tgt = idx + w * T;
        int64_t* st = tgt + w * T;
        check(ttk_memcpy_h2d(st, starts, static_cast<size_t>(w) * 8, stream()), "starts");
        check(ttk_gather_windows(tk->dev, st, w, T, idx, tgt, stream()), "gather windows");
        t->zero_grads();
        t->accumulate(idx, tgt, B, T, n_micro);
        t->optimizer_step(n_micro, lr);
        if (loss)
            check(ttk_memcpy_d2h(loss, t->loss_out, 4, stream()), "loss read");
        if (grad_norm)
            *grad_norm = t->ocfg.clip_norm > 0.0f ? t->opt->last_grad_norm() : 0.0f;
    });
}

float tt_lr_at(float base_lr, int64_t gstep, int64_t warmup, int64_t total_steps) {
    // apps/train.cpp:214-222, the same float expression order
    float lr_scale;
    if (gstep < warmup) {
        lr_scale = static_cast<float>(gstep + 1) / static_cast<float>(warmup);
    } else {
        const float prog = static_cast<float>(gstep - warmup) /
                           static_cast<float>(std::max<int64_t>(total_steps - warmup, 1));
        lr_scale = 0.1f + 0.9f * 0.5f * (1.0f + std::cos(3.14159265f * prog));
    }
    return base_lr * lr_scale;
}

int tt_trainer_save(void* h, const char* dir) {
    return guarded([&] {
        Trainer* t = T_(h);
        t->model->save_checkpoint(dir);
        // optimizer moments (host copies) and step count
        const size_t np = t->params.size();
        std::vector<std::vector<float>> host(2 * np);
        std::vector<std::pair<std::string, std::pair<int64_t, const float*>>> ts;
        for (size_t i = 0; i < np; ++i) {
            const int64_t n = t->params[i]->numel();
            for (int which = 0; which < 2; ++which) {
                auto& hb = host[2 * i + static_cast<size_t>(which)];
                hb.resize(static_cast<size_t>(n));
                check(ttk_memcpy_d2h(hb.data(), t->opt->moment(i, which),
                                     static_cast<size_t>(n) * 4, stream()),
                      "save: moments");
                ts.push_back({(which ? "v." : "m.") + std::to_string(i), {n, hb.data()}});
            }
        }
        const std::string meta = "{\"step\":\"" + std::to_string(t->opt->step_count()) + "\"}";
        write_safetensors(std::string(dir) + "/optimizer.safetensors", ts, meta);
    });
}

int tt_trainer_load(void* h, const char* dir) {
    return guarded([&] {
        Trainer* t = T_(h);
        t->drop_graph();
        t->model->load_checkpoint(dir);
        const std::string path = std::string(dir) + "/optimizer.safetensors";
        std::ifstream f(path, std::ios::binary);
        if (!f)
            return;  // weights-only checkpoint (e.g. written by the reference)
        const std::string hdr = read_header(f, path);
        const uint64_t base = 8 + hdr.size();
        int64_t step = 0;
        const size_t sp = hdr.find("\"step\":\"");
        if (sp == std::string::npos || std::sscanf(hdr.c_str() + sp, "\"step\":\"%ld", &step) != 1)
            throw std::runtime_error("load: optimizer step missing in " + path);
        std::vector<float> buf;
        for (size_t i = 0; i < t->params.size(); ++i) {
            const int64_t n = t->params[i]->numel();
            for (int which = 0; which < 2; ++which) {
                uint64_t beg = 0, end = 0;
                const std::string name = (which ? "v." : "m.") + std::to_string(i);
                if (!find_tensor(hdr, name, beg, end) || end - beg != static_cast<uint64_t>(n) * 4)
                    throw std::runtime_error("load: optimizer tensor " + name + " missing or resized");
                buf.resize(static_cast<size_t>(n));
                f.seekg(static_cast<std::streamoff>(base + beg), std::ios::beg);
                f.read(reinterpret_cast<char*>(buf.data()), static_cast<std::streamsize>(n * 4));
                if (!f)
                    throw std::runtime_error("load: read failed for " + name);
                check(ttk_memcpy_h2d(t->opt->moment(i, which), buf.data(),
                                     static_cast<size_t>(n) * 4, stream()),
                      "load: moments");
            }
        }
        check(ttk_stream_synchronize(stream()), "load");
        t->opt->set_step_count(step);
    });
}

int tt_plan_buckets(const int64_t* sizes, int n, int64_t bucket_bytes, int64_t* offsets,
                    int* bucket_of_param, int64_t* bucket_offset, int64_t* bucket_count,
                    int* n_buckets) {
    return guarded([&] {
        std::vector<int64_t> sz(sizes, sizes + n), offs;
        std::vector<Bucket> bk;
        std::vector<int> ids;
        plan_arena(sz, std::max<int64_t>(bucket_bytes / 4, 1), offs, bk, ids);
        for (int i = 0; i < n; ++i) {
            offsets[i] = offs[static_cast<size_t>(i)];
            bucket_of_param[i] = ids[static_cast<size_t>(i)];
        }
        for (size_t b = 0; b < bk.size(); ++b) {
            bucket_offset[b] = bk[b].offset;
            bucket_count[b] = bk[b].count;
        }
        *n_buckets = static_cast<int>(bk.size());
    });
}

int tt_trainer_comm_profile(void* h, int on) {
    return guarded([&] { T_(h)->comm_prof = on != 0; });
}

int tt_trainer_comm_stats(void* h, double* allreduce_ms, double* tail_ms, int64_t* n_allreduce,
                          int64_t* n_steps) {
    return guarded([&] {
        Trainer* t = T_(h);
        double busy = 0.0, tail = 0.0;
        for (auto& r : t->comm_recs) {
            float ms = 0.0f;
            check(ttk_event_synchronize(r.b), "event sync");
            check(ttk_event_elapsed_ms(r.a, r.b, &ms), "elapsed");
            busy += ms;
            t->event_pool.push_back(r.a), t->event_pool.push_back(r.b);
        }
        for (auto& r : t->tail_recs) {
            float ms = 0.0f;
            check(ttk_event_synchronize(r.b), "event sync");
            check(ttk_event_synchronize(r.a), "event sync");
            check(ttk_event_elapsed_ms(r.a, r.b, &ms), "elapsed");
            tail += ms > 0.0f ? ms : 0.0;
            t->event_pool.push_back(r.a), t->event_pool.push_back(r.b);
        }
        *allreduce_ms = busy;
        *tail_ms = tail;
        *n_allreduce = static_cast<int64_t>(t->comm_recs.size());
        *n_steps = static_cast<int64_t>(t->tail_recs.size());
        t->comm_recs.clear();
        t->tail_recs.clear();
    });
}

int tt_trainer_set_collective_timeout(void* h, double seconds) {
    return guarded([&] {
        if (!(seconds > 0.0))
            throw std::invalid_argument("collective timeout must be positive");
        T_(h)->coll_timeout_s = seconds;
    });
}

int tt_watchdog_selftest(int (*done)(void*), int (*async_error)(void*), int (*abort)(void*),
                         void* ctx, double timeout_s, int* outcome) {
    return guarded([&] {
        std::string why;
        *outcome = watch_collectives([&] { return done(ctx); }, [&] { return async_error(ctx); },
                                     [&] { abort(ctx); }, timeout_s, 1.0, why);
    });
}

int tt_trainer_dist_init(void* h, int rank, int world, const unsigned char id[128],
                         int64_t bucket_bytes) {
    return guarded([&] {
        Trainer* t = T_(h);
        t->drop_graph();  // the bucket plan below moves the gradient arena's layout
        check(ttk_dist_init(rank, world, id, &t->comm), "dist init");
        t->rank = rank;
        t->world = world;
        check(ttk_stream_create(&t->comm_stream), "comm stream");
        t->make_buckets(bucket_bytes > 0 ? bucket_bytes : (64ll << 20));
    });
}

}  // extern "C"
