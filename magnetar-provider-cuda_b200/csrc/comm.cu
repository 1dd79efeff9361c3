// Tensor-parallel group of one process per GPU over NCCL (NVLink 5 / NVSwitch).
//
// The reference sums a row-split projection's partial outputs by a serial reduce-to-root
// (P - 1 peer accumulates) followed by a serial copy back (P - 1 peer copies)
// (src/multi/tensor_parallel.rs:697-734, src/executor.rs:740-841).  Here every rank joins
// one NCCL communicator and the sum is a single in-place all-reduce.  The SwiGLU MLP entry
// point splits the down projection into row chunks: while chunk c+1 is multiplied on the
// compute stream, chunk c is all-reduced on a second stream, so the exchange overlaps the
// matmul.
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "internal.h"

// The communicator runs in NCCL's non-blocking mode: every NCCL call may return with its
// operation still in progress, and the host polls ncclCommGetAsyncError until it settles.  A
// rank that never joins, or a peer that died, therefore cannot block the host forever: after
// the group's timeout the communicator is aborted (ncclCommAbort) and the call fails with
// MG_DEVICE_UNAVAILABLE; an asynchronous NCCL error aborts it too (MG_DRIVER_FAILED).  An
// aborted communicator refuses further work.
struct mg_comm {
    mg::Device* device = nullptr;
    mg_device* handle = nullptr;
    ncclComm_t nccl = nullptr;
    int rank = 0, world = 1;
    cudaStream_t side = nullptr;  // all-reduce stream of the overlapped MLP
    std::vector<cudaEvent_t> events;
    int64_t timeout_ms = 300000;
    bool aborted = false;
    // mg_tp_mlp's timing events (mg_comm_set_mlp_timing): start, last down-projection chunk
    // done on the compute stream, the all-reduce stream joined.
    cudaEvent_t timing[3] = {nullptr, nullptr, nullptr};
    bool timed = false;
};

namespace mg {

// How a bounded settle ended.
enum SettleResult { kSettled = 0, kAsyncError = 1, kTimedOut = 2 };

// Polls `poll` (an NCCL result: ncclSuccess settled, ncclInProgress pending, anything else an
// error) until it settles or `timeout_ms` of host time pass, sleeping `sleep_us` between
// polls.  `abort` runs on an error or a timeout.  *polls counts the polls made.
static SettleResult settle_poll(int (*poll)(void*), void (*abort)(void*), void* ctx, int64_t timeout_ms,
                                int sleep_us, int* polls, int* last) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    *polls = 0;
    for (;;) {
        const int r = poll(ctx);
        (*polls)++;
        *last = r;
        if (r == (int)ncclSuccess) return kSettled;
        if (r != (int)ncclInProgress) {
            abort(ctx);
            return kAsyncError;
        }
        if (std::chrono::steady_clock::now() >= deadline) {
            abort(ctx);
            return kTimedOut;
        }
        if (sleep_us > 0) std::this_thread::sleep_for(std::chrono::microseconds(sleep_us));
    }
}

static int nccl_poll(void* ctx) {
    mg_comm* c = static_cast<mg_comm*>(ctx);
    ncclResult_t state = ncclSuccess;
    const ncclResult_t r = ncclCommGetAsyncError(c->nccl, &state);
    return r != ncclSuccess ? (int)r : (int)state;
}

static void nccl_abort(void* ctx) {
    mg_comm* c = static_cast<mg_comm*>(ctx);
    if (c->nccl && !c->aborted) ncclCommAbort(c->nccl);
    c->aborted = true;
    c->nccl = nullptr;
}

static mg_status settle_status(SettleResult res, int last, int64_t timeout_ms, const char* what) {
    if (res == kSettled) return MG_OK;
    if (res == kTimedOut)
        return fail(MG_DEVICE_UNAVAILABLE, "%s: the tensor-parallel group did not answer within %lld ms; the communicator was aborted",
                    what, (long long)timeout_ms);
    return fail(MG_DRIVER_FAILED, "%s: %s; the communicator was aborted", what, ncclGetErrorString((ncclResult_t)last));
}

// Waits, bounded, for the operation an NCCL call `r` started on `c` to be enqueued.
static mg_status comm_settle(mg_comm* c, ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl_abort(c);
        return fail(MG_DRIVER_FAILED, "%s: %s; the communicator was aborted", what, ncclGetErrorString(r));
    }
    int polls = 0, last = 0;
    const SettleResult res = settle_poll(nccl_poll, nccl_abort, c, c->timeout_ms, 50, &polls, &last);
    return settle_status(res, last, c->timeout_ms, what);
}

static mg_status comm_usable(mg_comm* c) {
    if (c->aborted) return fail(MG_DEVICE_UNAVAILABLE, "the tensor-parallel communicator was aborted");
    return MG_OK;
}

mg_status comm_all_reduce_buffer(mg_comm* c, Buffer* b) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    if (b->dtype != MG_F32) return fail(MG_DTYPE_UNSUPPORTED, "all-reduce sums f32 buffers only");
    MG_TRY(comm_usable(c));
    if (c->world == 1) return MG_OK;
    graph_touch(c->device, b->ptr);
    return comm_settle(c, ncclAllReduce(b->ptr, b->ptr, b->count, ncclFloat32, ncclSum, c->nccl, c->device->stream),
                       "all-reducing across the tensor-parallel group");
}

int comm_rank(mg_comm* c) { return c ? c->rank : 0; }
int comm_world(mg_comm* c) { return c ? c->world : 1; }

}  // namespace mg

using namespace mg;

namespace {
// Scripted NCCL states for the host-only settle test.
struct Script {
    const int* states;
    int n, at, aborted;
};
int script_poll(void* ctx) {
    Script* s = static_cast<Script*>(ctx);
    const int i = s->at < s->n ? s->at : s->n - 1;
    s->at++;
    return s->states[i];
}
void script_abort(void* ctx) { static_cast<Script*>(ctx)->aborted++; }
}  // namespace

extern "C" {

mg_status mg_comm_unique_id(unsigned char id[MG_COMM_ID_BYTES]) {
    if (!id) return fail(MG_INVALID_ARGUMENT, "null id");
    static_assert(sizeof(ncclUniqueId) == MG_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    const ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(MG_DRIVER_FAILED, "creating a communicator id: %s", ncclGetErrorString(r));
    memcpy(id, &u, sizeof u);
    return MG_OK;
}

mg_status mg_comm_init(mg_device* h, int rank, int world, const unsigned char id[MG_COMM_ID_BYTES], mg_comm** out) {
    MG_TRY(device_check(h));
    if (!id || !out) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (world < 1 || rank < 0 || rank >= world) return fail(MG_SHAPE_UNSUPPORTED, "rank %d of world %d", rank, world);
    mg_comm* c = new (std::nothrow) mg_comm();
    if (!c) return fail(MG_EXECUTION_FAILED, "host allocation failed");
    c->device = dev(h);
    c->handle = h;
    c->rank = rank;
    c->world = world;
    const char* t = getenv("MAGNETAR_CUDA_COMM_TIMEOUT_MS");
    if (t && atoll(t) > 0) c->timeout_ms = atoll(t);
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    if (world > 1) {
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        config.blocking = 0;
        const ncclResult_t r = ncclCommInitRankConfig(&c->nccl, world, u, rank, &config);
        mg_status s = comm_settle(c, r, "joining the tensor-parallel group");
        if (s != MG_OK) {
            delete c;
            return s;
        }
    }
    cudaError_t e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        if (c->nccl) ncclCommDestroy(c->nccl);
        delete c;
        return from_cuda(e, "creating the all-reduce stream");
    }
    device_ref(c->device);
    *out = c;
    return MG_OK;
}

mg_status mg_comm_destroy(mg_comm* c) {
    if (!c) return MG_OK;
    cudaSetDevice(c->device->ordinal);
    cudaStreamSynchronize(c->side);
    for (cudaEvent_t ev : c->events) cudaEventDestroy(ev);
    for (cudaEvent_t ev : c->timing)
        if (ev) cudaEventDestroy(ev);
    cudaStreamDestroy(c->side);
    if (c->nccl && !c->aborted) {
        // Non-blocking: the destroy itself may be in progress; bounded like every other call.
        ncclResult_t r = ncclCommFinalize(c->nccl);
        if (comm_settle(c, r, "finalizing the communicator") == MG_OK && c->nccl) ncclCommDestroy(c->nccl);
    }
    Device* d = c->device;
    delete c;
    device_unref(d);
    return MG_OK;
}

mg_status mg_comm_set_timeout(mg_comm* c, int64_t timeout_ms) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    if (timeout_ms <= 0) return fail(MG_INVALID_ARGUMENT, "a timeout must be positive");
    c->timeout_ms = timeout_ms;
    return MG_OK;
}

mg_status mg_comm_check(mg_comm* c) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    MG_TRY(comm_usable(c));
    if (!c->nccl) return MG_OK;
    const int r = nccl_poll(c);
    if (r == (int)ncclSuccess || r == (int)ncclInProgress) return MG_OK;
    nccl_abort(c);
    return fail(MG_DRIVER_FAILED, "the tensor-parallel group reported %s; the communicator was aborted",
                ncclGetErrorString((ncclResult_t)r));
}

mg_status mg_comm_abort(mg_comm* c) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    nccl_abort(c);
    return MG_OK;
}

int mg_comm_is_aborted(const mg_comm* c) { return c && c->aborted ? 1 : 0; }

mg_status mg_comm_wait(mg_comm* c, int64_t timeout_ms) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    MG_TRY(comm_usable(c));
    MG_TRY(device_check(c->handle));
    if (timeout_ms <= 0) timeout_ms = c->timeout_ms;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        const cudaError_t a = cudaStreamQuery(c->device->stream);
        const cudaError_t b = cudaStreamQuery(c->side);
        if (a != cudaSuccess && a != cudaErrorNotReady) return from_cuda(a, "waiting for the tensor-parallel step");
        if (b != cudaSuccess && b != cudaErrorNotReady) return from_cuda(b, "waiting for the tensor-parallel step");
        if (c->nccl) {
            const int r = nccl_poll(c);
            if (r != (int)ncclSuccess && r != (int)ncclInProgress) {
                nccl_abort(c);
                return fail(MG_DRIVER_FAILED, "the tensor-parallel group reported %s; the communicator was aborted",
                            ncclGetErrorString((ncclResult_t)r));
            }
        }
        if (a == cudaSuccess && b == cudaSuccess) return MG_OK;
        if (std::chrono::steady_clock::now() >= deadline) {
            nccl_abort(c);
            return fail(MG_DEVICE_UNAVAILABLE, "the tensor-parallel step did not finish within %lld ms; the communicator was aborted",
                        (long long)timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

mg_status mg_comm_settle_selftest(const int* states, int count, int64_t timeout_ms, int* aborted, int* polls) {
    if (!states || count < 1 || !aborted || !polls) return fail(MG_INVALID_ARGUMENT, "null argument");
    Script sc{states, count, 0, 0};
    int last = 0;
    const SettleResult res = settle_poll(script_poll, script_abort, &sc, timeout_ms, 100, polls, &last);
    *aborted = sc.aborted;
    return settle_status(res, last, timeout_ms, "settling a scripted operation");
}

mg_status mg_comm_all_reduce(mg_comm* c, mg_buffer* b) {
    if (!c || !b) return fail(MG_INVALID_ARGUMENT, "null argument");
    MG_TRY(device_check(c->handle));
    return comm_all_reduce_buffer(c, buf(b));
}

mg_status mg_tp_mlp(mg_comm* c, const mg_buffer* xh, const mg_buffer* gh, const mg_buffer* uh, const mg_buffer* dh,
                    int chunks, mg_buffer** out) {
    if (!c || !xh || !gh || !uh || !dh || !out) return fail(MG_INVALID_ARGUMENT, "null argument");
    MG_TRY(device_check(c->handle));
    MG_TRY(comm_usable(c));
    Device* d = c->device;
    const Buffer* x = buf(xh);
    const Buffer* dn = buf(dh);
    if (x->rank != 2 || dn->rank != 2) return fail(MG_SHAPE_UNSUPPORTED, "the MLP takes rank-2 activations and weights");
    const bool timed = c->timing[0] != nullptr;
    c->timed = false;
    if (timed) MG_CUDA(cudaEventRecord(c->timing[0], d->stream), "recording the MLP's start");
    // h = silu(x G_s) * (x U_s): [tokens, ffn_share], from the rank's column shards.
    mg_buffer* hh = nullptr;
    MG_TRY(mg_gated_matmul(c->handle, xh, gh, uh, 0, 0, &hh));
    Buffer* hb = buf(hh);
    const uint64_t tokens = hb->shape[0], share = hb->shape[1];
    if (dn->shape[0] != share) {
        buffer_free(hb);
        return fail(MG_SHAPE_UNSUPPORTED, "down shard has %llu rows, the gate/up shards give %llu columns",
                    (unsigned long long)dn->shape[0], (unsigned long long)share);
    }
    const uint64_t hidden = dn->shape[1];
    const uint64_t shape[2] = {tokens, hidden};
    Buffer* y;
    mg_status s = output_for(d, MG_F32, 2, shape, out, &y);
    if (s != MG_OK) {
        buffer_free(hb);
        return s;
    }
    if (chunks < 1) chunks = 1;
    if ((uint64_t)chunks > tokens) chunks = (int)(tokens ? tokens : 1);
    while ((int)c->events.size() < chunks + 1) {
        cudaEvent_t ev;
        cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            buffer_free(hb);
            return from_cuda(e, "creating an event");
        }
        c->events.push_back(ev);
    }
    // y_c = h[rows_c] D_s, then the sum over ranks of chunk c on the side stream while the
    // next chunk multiplies.
    const uint64_t per = (tokens + chunks - 1) / chunks;
    for (int i = 0; i < chunks && s == MG_OK; i++) {
        const uint64_t r0 = (uint64_t)i * per, r1 = r0 + per < tokens ? r0 + per : tokens;
        if (r0 >= r1) break;
        k::GemmArgs g{};
        g.a = (const float*)hb->ptr + r0 * share;
        g.b = (const float*)dn->ptr;
        g.out = (float*)y->ptr + r0 * hidden;
        g.m = r1 - r0;
        g.n = hidden;
        g.k = share;
        s = k::gemm(d, g);
        if (s != MG_OK || c->world == 1) continue;
        cudaError_t e = cudaEventRecord(c->events[i], d->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->side, c->events[i], 0);
        if (e != cudaSuccess) {
            s = from_cuda(e, "ordering the chunked all-reduce");
            break;
        }
        s = comm_settle(c, ncclAllReduce(g.out, g.out, (r1 - r0) * hidden, ncclFloat32, ncclSum, c->nccl, c->side),
                        "all-reducing an MLP chunk");
    }
    if (timed && s == MG_OK) {
        cudaError_t e = cudaEventRecord(c->timing[1], d->stream);
        if (e != cudaSuccess) s = from_cuda(e, "recording the MLP's compute end");
    }
    if (c->world > 1) {
        cudaError_t e = cudaEventRecord(c->events[chunks], c->side);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(d->stream, c->events[chunks], 0);
        if (e != cudaSuccess && s == MG_OK) s = from_cuda(e, "joining the all-reduce stream");
    }
    if (timed && s == MG_OK) {
        cudaError_t e = cudaEventRecord(c->timing[2], d->stream);
        if (e != cudaSuccess) s = from_cuda(e, "recording the MLP's end");
        else c->timed = true;
    }
    buffer_free(hb);
    return s;
}

mg_status mg_comm_set_mlp_timing(mg_comm* c, int on) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    MG_TRY(device_check(c->handle));
    for (cudaEvent_t& ev : c->timing) {
        if (on && !ev) MG_CUDA(cudaEventCreate(&ev), "creating a timing event");
        if (!on && ev) {
            cudaEventDestroy(ev);
            ev = nullptr;
        }
    }
    c->timed = false;
    return MG_OK;
}

mg_status mg_comm_mlp_timing(mg_comm* c, float* compute_ms, float* exposed_ms) {
    if (!c || !compute_ms || !exposed_ms) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (!c->timed) return fail(MG_INVALID_ARGUMENT, "no timed MLP call since timing was switched on");
    MG_TRY(device_check(c->handle));
    MG_CUDA(cudaEventSynchronize(c->timing[2]), "waiting for the timed MLP");
    MG_CUDA(cudaEventElapsedTime(compute_ms, c->timing[0], c->timing[1]), "reading the MLP's compute time");
    MG_CUDA(cudaEventElapsedTime(exposed_ms, c->timing[1], c->timing[2]), "reading the MLP's exposed all-reduce");
    return MG_OK;
}

}  // extern "C"
