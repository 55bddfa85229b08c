/* b2s_server.h -- batched data-parallel serving of BitVLA-shape observations over several GPUs (C ABI).
 *
 * Replaces the reference model-server's serialization of every prediction behind one global mutex
 * (robot_server/session.cpp:124, `std::unique_lock<std::mutex> lock(predict_mutex)` around
 * policy.predict) with one engine per GPU and a bounded request queue: any number of client threads submit
 * observations; each engine's worker thread takes up to max_batch waiting requests at once (FIFO), runs
 * them as one batched forward on its own GPU, and completes each request with its actions or with the
 * engine's error status. The wire protocol in front of it is unchanged (robot_server/protocol.h:11-87);
 * this is what a session calls instead of policy.predict.
 *
 * Failure handling: an engine whose predict call fails completes the requests of that batch with its
 * status and message, is marked unhealthy and takes no further requests; the other engines keep serving
 * the queue. When no healthy engine is left, waiting and newly submitted requests fail with
 * B2S_ERR_UNAVAILABLE.
 *
 * Threading: every function is thread-safe except b2s_server_free, which must not race with other calls on
 * the same server. A request id is waited for exactly once.
 */
#ifndef B2S_SERVER_H
#define B2S_SERVER_H

#include <stddef.h>
#include <stdint.h>

#include "b2s_bitvla.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B2S_ERR_BUSY (-7)        /* the request queue is full */
#define B2S_ERR_UNAVAILABLE (-8) /* no healthy engine is left */
#define B2S_ERR_TIMEOUT (-9)     /* b2s_server_wait ran out of time (the request stays pending) */

typedef struct b2s_server b2s_server;

/* One engine (normally one GPU). `predict` runs `batch` observations -- images [batch][image_bytes] (HWC
 * uint8), tokens [batch][n_text] -- and writes actions [batch][action_floats]; it returns B2S_OK or a
 * negative status (its message is taken from b2s_last_error() on the worker thread). It is only ever called
 * from the engine's own worker thread. `setup` (may be NULL) runs once on that thread before the first
 * predict (e.g. to make the engine's device current and build the model); a failing setup marks the engine
 * unhealthy. `destroy` (may be NULL) runs on the worker thread when the server is freed. */
typedef struct b2s_engine_ops {
    int (*setup)(void *engine);
    int (*predict)(void *engine, int batch, const uint8_t *images, const int32_t *tokens, float *actions);
    void (*destroy)(void *engine);
} b2s_engine_ops;

typedef struct b2s_server_shape {
    int image_bytes;    /* bytes of one observation's HWC uint8 image */
    int n_text;         /* token ids per observation */
    int action_floats;  /* floats of one observation's actions */
} b2s_server_shape;

/* For engine implementations: records `msg` as the message of this thread's failing call (what the waiter of
 * each request of the batch receives from b2s_last_error()) and returns `status`. */
int b2s_server_engine_error(int status, const char *msg);

/* A server over `n_engines` caller-provided engines sharing `ops`; max_batch observations per engine call,
 * at most queue_capacity requests waiting. The worker threads start (and run setup) before this returns;
 * engines whose setup failed are reported by b2s_server_engine_status. */
int b2s_server_create(const b2s_engine_ops *ops, void *const *engines, int n_engines, const b2s_server_shape *shape,
                      int max_batch, int queue_capacity, b2s_server **out);

/* A server with one BitVLA-shape engine per listed CUDA device, each a b2s_bitvla model built on its
 * device from `seed` (b2s_bitvla_create) or, when gguf_path is not NULL, from that file, with its own
 * stream; engine calls are b2s_bitvla_predict. */
int b2s_server_create_bitvla(const int *devices, int n_devices, const b2s_bitvla_config *cfg, uint32_t seed,
                             const char *gguf_path, int max_batch, int queue_capacity, b2s_server **out);

/* Queues one observation (the image and tokens are copied). Returns a request id >= 0, or a negative status
 * (B2S_ERR_BUSY when queue_capacity requests are already waiting, B2S_ERR_UNAVAILABLE when no engine is
 * healthy, B2S_ERR_INVALID_ARG). */
int64_t b2s_server_submit(b2s_server *s, const uint8_t *image_hwc, const int32_t *tokens);

/* Waits for request `id` (timeout_ms < 0: no limit) and copies its actions (action_floats floats) to
 * `actions`. Returns the request's status: B2S_OK, the failing engine's status (message in b2s_last_error()
 * of this thread), B2S_ERR_UNAVAILABLE, or B2S_ERR_TIMEOUT (the request stays pending and may be waited for
 * again). On completion *latency_ms (may be NULL) is the time from submit to completion and *engine (may
 * be NULL) the index of the engine that ran it (-1 if none did). */
int b2s_server_wait(b2s_server *s, int64_t id, float *actions, int timeout_ms, double *latency_ms, int *engine);

/* Number of engines; per engine: 1 healthy / 0 unhealthy, and the requests it completed. */
int b2s_server_engines(const b2s_server *s);
int b2s_server_engine_status(const b2s_server *s, int engine, int *healthy, int64_t *completed, int64_t *batches);

/* Stops the workers (requests still waiting fail with B2S_ERR_UNAVAILABLE), destroys the engines, frees. */
void b2s_server_free(b2s_server *s);

#ifdef __cplusplus
}
#endif
#endif /* B2S_SERVER_H */
