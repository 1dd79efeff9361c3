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

#include <cstring>
#include <new>
#include <vector>

#include "internal.h"

struct mg_comm {
    mg::Device* device = nullptr;
    mg_device* handle = nullptr;
    ncclComm_t nccl = nullptr;
    int rank = 0, world = 1;
    cudaStream_t side = nullptr;  // all-reduce stream of the overlapped MLP
    std::vector<cudaEvent_t> events;
};

namespace mg {

static mg_status from_nccl(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return MG_OK;
    return fail(MG_DRIVER_FAILED, "%s: %s", what, ncclGetErrorString(r));
}

mg_status comm_all_reduce_buffer(mg_comm* c, Buffer* b) {
    if (!c) return fail(MG_INVALID_ARGUMENT, "null communicator");
    if (b->dtype != MG_F32) return fail(MG_DTYPE_UNSUPPORTED, "all-reduce sums f32 buffers only");
    if (c->world == 1) return MG_OK;
    return from_nccl(ncclAllReduce(b->ptr, b->ptr, b->count, ncclFloat32, ncclSum, c->nccl, c->device->stream),
                     "all-reducing across the tensor-parallel group");
}

int comm_rank(mg_comm* c) { return c ? c->rank : 0; }
int comm_world(mg_comm* c) { return c ? c->world : 1; }

}  // namespace mg

using namespace mg;

extern "C" {

mg_status mg_comm_unique_id(unsigned char id[MG_COMM_ID_BYTES]) {
    if (!id) return fail(MG_INVALID_ARGUMENT, "null id");
    static_assert(sizeof(ncclUniqueId) == MG_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    MG_TRY(from_nccl(ncclGetUniqueId(&u), "creating a communicator id"));
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
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    if (world > 1) {
        mg_status s = from_nccl(ncclCommInitRank(&c->nccl, world, u, rank), "joining the tensor-parallel group");
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
    cudaStreamDestroy(c->side);
    if (c->nccl) ncclCommDestroy(c->nccl);
    Device* d = c->device;
    delete c;
    device_unref(d);
    return MG_OK;
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
    Device* d = c->device;
    const Buffer* x = buf(xh);
    const Buffer* dn = buf(dh);
    if (x->rank != 2 || dn->rank != 2) return fail(MG_SHAPE_UNSUPPORTED, "the MLP takes rank-2 activations and weights");
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
        s = from_nccl(ncclAllReduce(g.out, g.out, (r1 - r0) * hidden, ncclFloat32, ncclSum, c->nccl, c->side),
                      "all-reducing an MLP chunk");
    }
    if (c->world > 1) {
        cudaError_t e = cudaEventRecord(c->events[chunks], c->side);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(d->stream, c->events[chunks], 0);
        if (e != cudaSuccess && s == MG_OK) s = from_cuda(e, "joining the all-reduce stream");
    }
    buffer_free(hb);
    return s;
}

}  // extern "C"
