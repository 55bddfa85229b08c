// server.cu -- batched data-parallel serving over several engines (C ABI in include/b2s_server.h).
//
// The reference model-server runs every prediction under one global mutex (robot_server/session.cpp:124)
// behind one accept loop (robot_server/model-server.cpp:239-253), so a second GPU or a second waiting
// client gains nothing. Here each engine (normally one GPU holding a full weight replica) has a worker
// thread; client threads submit single observations into one bounded FIFO queue; a worker that becomes
// free takes up to max_batch waiting requests at once and runs them as one batched forward. Observations
// are independent, so engines never communicate: there is no collective anywhere on this path.
//
// Failure handling follows the reference's status-plus-message convention (session.cpp:132-135 sends
// status_internal_error with the message): a failing engine call completes its batch's requests with the
// engine's status and message, the engine is marked unhealthy and stops taking requests, and the others
// keep serving. With no healthy engine left, queued and new requests fail with B2S_ERR_UNAVAILABLE.
#include <cuda_runtime.h>

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "b2s.h"
#include "b2s_bitvla.h"
#include "b2s_internal.h"
#include "b2s_server.h"

namespace {

using Clock = std::chrono::steady_clock;

struct Request {
    std::vector<uint8_t> image;
    std::vector<int32_t> tokens;
    std::vector<float> actions;
    bool done = false;
    int status = B2S_OK;
    int engine = -1;
    std::string msg;
    Clock::time_point t_submit, t_done;
};

struct Engine {
    void* ctx = nullptr;
    std::thread th;
    bool healthy = true;
    int64_t completed = 0, batches = 0;
};

// A BitVLA-shape model on one device (the engine of b2s_server_create_bitvla).
struct BitvlaEngine {
    int device = 0;
    b2s_bitvla_config cfg{};
    uint32_t seed = 0;
    std::string gguf;
    int max_batch = 1;
    b2s_bitvla* model = nullptr;
    cudaStream_t stream = nullptr;
};

int bitvla_setup(void* p) {
    BitvlaEngine* e = static_cast<BitvlaEngine*>(p);
    cudaError_t ce = cudaSetDevice(e->device);
    if (ce != cudaSuccess) return b2s::set_last_error(B2S_ERR_CUDA, cudaGetErrorString(ce));
    int rc = e->gguf.empty() ? b2s_bitvla_create(&e->cfg, e->seed, e->max_batch, &e->model)
                             : b2s_bitvla_create_from_gguf(e->gguf.c_str(), e->max_batch, &e->model);
    if (rc) return rc;
    ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (ce != cudaSuccess) return b2s::set_last_error(B2S_ERR_CUDA, cudaGetErrorString(ce));
    return B2S_OK;
}

int bitvla_predict(void* p, int batch, const uint8_t* images, const int32_t* tokens, float* actions) {
    BitvlaEngine* e = static_cast<BitvlaEngine*>(p);
    return b2s_bitvla_predict(e->model, batch, images, tokens, actions, e->stream);
}

void bitvla_destroy(void* p) {
    BitvlaEngine* e = static_cast<BitvlaEngine*>(p);
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamDestroy(e->stream);
    b2s_bitvla_free(e->model);
    e->model = nullptr;
    e->stream = nullptr;
}

}  // namespace

struct b2s_server {
    b2s_engine_ops ops{};
    b2s_server_shape shape{};
    int max_batch = 1, capacity = 1;
    std::mutex mu;
    std::condition_variable cv_work, cv_done;
    std::deque<std::shared_ptr<Request>> queue;
    std::unordered_map<int64_t, std::shared_ptr<Request>> requests;
    int64_t next_id = 0;
    bool stop = false;
    int healthy = 0, setups_pending = 0;
    std::vector<Engine> engines;
    std::vector<std::unique_ptr<BitvlaEngine>> owned;  // engines built by b2s_server_create_bitvla

    // Completes every queued request with B2S_ERR_UNAVAILABLE (caller holds mu).
    void fail_queue_locked(const char* why) {
        const Clock::time_point now = Clock::now();
        for (auto& r : queue) {
            r->status = B2S_ERR_UNAVAILABLE;
            r->msg = why;
            r->done = true;
            r->t_done = now;
        }
        queue.clear();
        cv_done.notify_all();
    }

    void mark_unhealthy_locked(Engine& e) {
        if (!e.healthy) return;
        e.healthy = false;
        if (--healthy == 0) fail_queue_locked("no healthy engine is left");
    }

    void worker(int idx) {
        Engine& E = engines[(size_t)idx];
        int rc = ops.setup ? ops.setup(E.ctx) : B2S_OK;
        {
            std::lock_guard<std::mutex> lk(mu);
            if (rc) mark_unhealthy_locked(E);
            --setups_pending;
            cv_done.notify_all();
        }
        const size_t ib = (size_t)shape.image_bytes, nt = (size_t)shape.n_text, na = (size_t)shape.action_floats;
        std::vector<uint8_t> img((size_t)max_batch * ib);
        std::vector<int32_t> tok((size_t)max_batch * (nt ? nt : 1));
        std::vector<float> act((size_t)max_batch * na);
        while (rc == B2S_OK) {
            std::vector<std::shared_ptr<Request>> batch;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv_work.wait(lk, [&] { return stop || !queue.empty(); });
                if (stop) break;
                while (!queue.empty() && (int)batch.size() < max_batch) {
                    batch.push_back(queue.front());
                    queue.pop_front();
                }
            }
            const int n = (int)batch.size();
            for (int i = 0; i < n; ++i) {
                memcpy(img.data() + (size_t)i * ib, batch[(size_t)i]->image.data(), ib);
                if (nt) memcpy(tok.data() + (size_t)i * nt, batch[(size_t)i]->tokens.data(), nt * sizeof(int32_t));
            }
            rc = ops.predict(E.ctx, n, img.data(), tok.data(), act.data());
            const std::string msg = rc ? std::string(b2s_last_error()) : std::string();
            std::lock_guard<std::mutex> lk(mu);
            const Clock::time_point now = Clock::now();
            for (int i = 0; i < n; ++i) {
                Request& r = *batch[(size_t)i];
                r.status = rc;
                r.msg = msg;
                r.engine = idx;
                if (!rc) r.actions.assign(act.begin() + (ptrdiff_t)(i * na), act.begin() + (ptrdiff_t)((i + 1) * na));
                r.done = true;
                r.t_done = now;
            }
            E.completed += n;
            E.batches += 1;
            if (rc) mark_unhealthy_locked(E);
            cv_done.notify_all();
        }
        // Engines are destroyed on their own thread, once the server is stopping.
        {
            std::unique_lock<std::mutex> lk(mu);
            cv_work.wait(lk, [&] { return stop; });
        }
        if (ops.destroy) ops.destroy(E.ctx);
    }
};

namespace {

int start(b2s_server* s, void* const* engines, int n) {
    s->engines.resize((size_t)n);
    s->healthy = n;
    s->setups_pending = n;
    for (int i = 0; i < n; ++i) s->engines[(size_t)i].ctx = engines[i];
    for (int i = 0; i < n; ++i) s->engines[(size_t)i].th = std::thread([s, i] { s->worker(i); });
    std::unique_lock<std::mutex> lk(s->mu);
    s->cv_done.wait(lk, [&] { return s->setups_pending == 0; });
    if (s->healthy == 0) return b2s::set_last_error(B2S_ERR_UNAVAILABLE, "server: no engine finished its setup");
    return B2S_OK;
}

}  // namespace

extern "C" {

int b2s_server_create(const b2s_engine_ops* ops, void* const* engines, int n_engines, const b2s_server_shape* shape,
                      int max_batch, int queue_capacity, b2s_server** out) {
    if (!out) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create: out is NULL");
    *out = nullptr;
    if (!ops || !ops->predict || !engines || n_engines <= 0 || !shape || shape->image_bytes <= 0 ||
        shape->n_text < 0 || shape->action_floats <= 0 || max_batch <= 0 || queue_capacity <= 0)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create: bad arguments");
    b2s_server* s = new (std::nothrow) b2s_server();
    if (!s) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create: out of host memory");
    s->ops = *ops;
    s->shape = *shape;
    s->max_batch = max_batch;
    s->capacity = queue_capacity;
    const int rc = start(s, engines, n_engines);
    if (rc) {
        const std::string msg = b2s_last_error();
        b2s_server_free(s);
        return b2s::set_last_error(rc, msg.c_str());
    }
    *out = s;
    return B2S_OK;
}

int b2s_server_create_bitvla(const int* devices, int n_devices, const b2s_bitvla_config* cfg, uint32_t seed,
                             const char* gguf_path, int max_batch, int queue_capacity, b2s_server** out) {
    if (!out) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create_bitvla: out is NULL");
    *out = nullptr;
    if (!devices || n_devices <= 0 || (!cfg && !gguf_path) || max_batch <= 0 || queue_capacity <= 0)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create_bitvla: bad arguments");
    b2s_bitvla_config c;
    b2s_bitvla_default_config(&c);
    if (cfg) c = *cfg;
    if (gguf_path && !cfg) {  // the shape comes from the file: read it from a one-observation model
        b2s_bitvla* probe = nullptr;
        int rc = b2s_bitvla_create_from_gguf(gguf_path, 1, &probe);
        if (!rc) rc = b2s_bitvla_get_config(probe, &c);
        b2s_bitvla_free(probe);
        if (rc) return rc;
    }
    b2s_server* s = new (std::nothrow) b2s_server();
    if (!s) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_create_bitvla: out of host memory");
    s->ops.setup = bitvla_setup;
    s->ops.predict = bitvla_predict;
    s->ops.destroy = bitvla_destroy;
    const int g = c.image_size;
    s->shape.image_bytes = 3 * g * g;
    s->shape.n_text = c.n_text;
    s->shape.action_floats = c.action_chunk * c.action_dim;
    s->max_batch = max_batch;
    s->capacity = queue_capacity;
    std::vector<void*> ctx;
    for (int i = 0; i < n_devices; ++i) {
        std::unique_ptr<BitvlaEngine> e(new BitvlaEngine());
        e->device = devices[i];
        e->cfg = c;
        e->seed = seed;
        e->gguf = gguf_path ? gguf_path : "";
        e->max_batch = max_batch;
        ctx.push_back(e.get());
        s->owned.push_back(std::move(e));
    }
    const int rc = start(s, ctx.data(), n_devices);
    if (rc) {
        const std::string msg = b2s_last_error();
        b2s_server_free(s);
        return b2s::set_last_error(rc, msg.c_str());
    }
    *out = s;
    return B2S_OK;
}

int64_t b2s_server_submit(b2s_server* s, const uint8_t* image_hwc, const int32_t* tokens) {
    if (!s || !image_hwc || (!tokens && s->shape.n_text > 0))
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_submit: bad arguments");
    auto r = std::make_shared<Request>();
    r->image.assign(image_hwc, image_hwc + s->shape.image_bytes);
    if (s->shape.n_text > 0) r->tokens.assign(tokens, tokens + s->shape.n_text);
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->stop || s->healthy == 0) return b2s::set_last_error(B2S_ERR_UNAVAILABLE, "server_submit: no healthy engine");
    if ((int)s->queue.size() >= s->capacity)
        return b2s::set_last_error(B2S_ERR_BUSY, "server_submit: request queue is full");
    const int64_t id = s->next_id++;
    r->t_submit = Clock::now();
    s->requests.emplace(id, r);
    s->queue.push_back(r);
    s->cv_work.notify_one();
    return id;
}

int b2s_server_wait(b2s_server* s, int64_t id, float* actions, int timeout_ms, double* latency_ms, int* engine) {
    if (!s || !actions) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_wait: bad arguments");
    std::unique_lock<std::mutex> lk(s->mu);
    auto it = s->requests.find(id);
    if (it == s->requests.end()) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_wait: unknown request id");
    std::shared_ptr<Request> r = it->second;
    if (timeout_ms < 0) {
        s->cv_done.wait(lk, [&] { return r->done; });
    } else if (!s->cv_done.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return r->done; })) {
        return b2s::set_last_error(B2S_ERR_TIMEOUT, "server_wait: timed out (the request is still pending)");
    }
    s->requests.erase(it);
    if (latency_ms) latency_ms[0] = std::chrono::duration<double, std::milli>(r->t_done - r->t_submit).count();
    if (engine) engine[0] = r->engine;
    if (r->status != B2S_OK) return b2s::set_last_error(r->status, r->msg.c_str());
    memcpy(actions, r->actions.data(), sizeof(float) * r->actions.size());
    return B2S_OK;
}

int b2s_server_engine_error(int status, const char* msg) { return b2s::set_last_error(status, msg ? msg : ""); }

int b2s_server_engines(const b2s_server* s) { return s ? (int)s->engines.size() : 0; }

int b2s_server_engine_status(const b2s_server* s, int engine, int* healthy, int64_t* completed, int64_t* batches) {
    if (!s || engine < 0 || engine >= (int)s->engines.size())
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "server_engine_status: bad engine index");
    b2s_server* m = const_cast<b2s_server*>(s);
    std::lock_guard<std::mutex> lk(m->mu);
    const Engine& e = s->engines[(size_t)engine];
    if (healthy) *healthy = e.healthy ? 1 : 0;
    if (completed) *completed = e.completed;
    if (batches) *batches = e.batches;
    return B2S_OK;
}

void b2s_server_free(b2s_server* s) {
    if (!s) return;
    {
        std::lock_guard<std::mutex> lk(s->mu);
        s->stop = true;
        s->fail_queue_locked("server is shutting down");
        s->cv_work.notify_all();
    }
    for (auto& e : s->engines)
        if (e.th.joinable()) e.th.join();
    delete s;
}

}  // extern "C"
