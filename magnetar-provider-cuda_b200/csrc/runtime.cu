// Device, buffer and error plumbing behind the C ABI.
//
// Replaces the reference's cudarc context/stream per GPU (src/kernels.rs:795-857,
// src/device.rs:41-92) and its CudaDeviceBuffer allocations: one stream per device, and a
// dedicated stream-ordered memory pool (cudaMallocAsync) whose release threshold keeps freed
// blocks for reuse, so chained kernels allocate without synchronising.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>

#include "internal.h"

namespace mg {

static thread_local std::string t_last_error;

mg_status fail(mg_status status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

void clear_error() { t_last_error.clear(); }

// src/error.rs:71-91: out of memory and missing devices keep their categories, every
// other driver failure is DriverFailed.  The detail is the runtime's error text only.
mg_status from_cuda(cudaError_t err, const char* what) {
    mg_status s = MG_DRIVER_FAILED;
    if (err == cudaErrorMemoryAllocation) s = MG_OUT_OF_DEVICE_MEMORY;
    else if (err == cudaErrorNoDevice || err == cudaErrorInvalidDevice || err == cudaErrorInsufficientDriver)
        s = MG_DEVICE_UNAVAILABLE;
    else if (err == cudaErrorStreamCaptureUnsupported || err == cudaErrorStreamCaptureInvalidated ||
             err == cudaErrorStreamCaptureUnjoined || err == cudaErrorStreamCaptureIsolation ||
             err == cudaErrorStreamCaptureImplicit || err == cudaErrorCapturedEvent)
        s = MG_CAPTURE_UNSUPPORTED;
    return fail(s, "%s: %s", what, cudaGetErrorString(err));
}

const char* dtype_name(mg_dtype t) {
    switch (t) {
        case MG_F32: return "f32";
        case MG_F16: return "f16";
        case MG_BF16: return "bf16";
        case MG_Q8_0: return "q8_0";
    }
    return "?";
}

std::string shape_str(const Buffer* b) {
    std::string s = "[";
    for (int i = 0; i < b->rank; i++) {
        if (i) s += ", ";
        s += std::to_string(b->shape[i]);
    }
    return s + "]";
}

bool same_shape(const Buffer* a, const Buffer* b) {
    if (a->rank != b->rank) return false;
    for (int i = 0; i < a->rank; i++)
        if (a->shape[i] != b->shape[i]) return false;
    return true;
}

mg_status device_check(mg_device* d) {
    if (!d) return fail(MG_INVALID_ARGUMENT, "null device handle");
    if (dev(d)->closed.load()) return fail(MG_DEVICE_UNAVAILABLE, "the device handle was closed");
    cudaError_t e = cudaSetDevice(dev(d)->ordinal);
    if (e != cudaSuccess) return from_cuda(e, "selecting the device");
    return MG_OK;
}

mg_status device_alloc(Device* d, size_t bytes, void** ptr) {
    *ptr = nullptr;
    if (bytes == 0) bytes = 16;  // a device buffer is never empty (src/kernels.rs:4454-4455)
    cudaError_t e;
    if (d->capturing) {
        e = cudaMalloc(ptr, bytes);
        if (e == cudaSuccess) {
            std::lock_guard<std::mutex> g(d->mem_lock);
            d->plain_allocs.insert(*ptr);
            d->capture_touched.insert(*ptr);
        }
    } else {
        e = cudaMallocFromPoolAsync(ptr, bytes, d->pool, d->stream);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return fail(e == cudaErrorMemoryAllocation ? MG_OUT_OF_DEVICE_MEMORY : MG_DRIVER_FAILED,
                    "allocating %zu bytes on cuda:%d: %s", bytes, d->ordinal, cudaGetErrorString(e));
    }
    return MG_OK;
}

// Frees `ptr` now (in stream order for pool blocks).  Caller holds mem_lock.
static void free_now(Device* d, void* ptr) {
    auto it = d->plain_allocs.find(ptr);
    if (it != d->plain_allocs.end()) {
        d->plain_allocs.erase(it);
        cudaFree(ptr);
    } else {
        cudaFreeAsync(ptr, d->stream);
    }
}

void device_free(Device* d, void* ptr) {
    if (!ptr) return;
    std::lock_guard<std::mutex> g(d->mem_lock);
    if (d->capturing) {
        d->deferred_frees.push_back(ptr);
        return;
    }
    if (d->graph_refs.count(ptr)) {  // a live captured step still addresses it
        d->held_frees.insert(ptr);
        return;
    }
    free_now(d, ptr);
}

void flush_deferred_frees(Device* d) {
    std::vector<void*> pending;
    {
        std::lock_guard<std::mutex> g(d->mem_lock);
        pending.swap(d->deferred_frees);
    }
    for (void* p : pending) device_free(d, p);
}

void graph_touch(Device* d, const void* ptr) {
    if (!ptr || !d->capturing) return;
    std::lock_guard<std::mutex> g(d->mem_lock);
    d->capture_touched.insert(const_cast<void*>(ptr));
}

std::vector<void*> graph_take(Device* d) {
    std::lock_guard<std::mutex> g(d->mem_lock);
    std::vector<void*> v(d->capture_touched.begin(), d->capture_touched.end());
    d->capture_touched.clear();
    return v;
}

void graph_hold(Device* d, const std::vector<void*>& blocks) {
    std::lock_guard<std::mutex> g(d->mem_lock);
    for (void* p : blocks) d->graph_refs[p]++;
}

void graph_release(Device* d, const std::vector<void*>& blocks) {
    std::lock_guard<std::mutex> g(d->mem_lock);
    for (void* p : blocks) {
        auto it = d->graph_refs.find(p);
        if (it == d->graph_refs.end()) continue;
        if (--it->second > 0) continue;
        d->graph_refs.erase(it);
        auto h = d->held_frees.find(p);
        if (h != d->held_frees.end()) {
            d->held_frees.erase(h);
            free_now(d, p);
        }
    }
}

// ---- scratch workspaces -------------------------------------------------------------------
// Slots are grown on demand and freed in stream order, so a later kernel on the same stream
// may reuse a workspace as soon as the previous user's kernels are ordered before it.  A
// workspace a captured step addresses is recorded for that step: when the slot grows later,
// the old block stays allocated until every step that addresses it is released.
mg_status scratch(Device* d, int slot, size_t bytes, void** ptr) {
    if (d->scratch_bytes[slot] < bytes) {
        // The old workspace is released in stream order (or, during a capture, once the
        // capture ends, since earlier captured kernels still address it).
        if (d->scratch_ptr[slot]) device_free(d, d->scratch_ptr[slot]);
        d->scratch_ptr[slot] = nullptr;
        d->scratch_bytes[slot] = 0;
        size_t grow = bytes + bytes / 4;
        MG_TRY(device_alloc(d, grow, &d->scratch_ptr[slot]));
        d->scratch_bytes[slot] = grow;
    }
    *ptr = d->scratch_ptr[slot];
    graph_touch(d, *ptr);
    return MG_OK;
}

static void scratch_release(Device* d) {
    for (int i = 0; i < 8; i++) {
        if (d->scratch_ptr[i]) device_free(d, d->scratch_ptr[i]);
        d->scratch_ptr[i] = nullptr;
        d->scratch_bytes[i] = 0;
    }
}

// ---- buffers --------------------------------------------------------------------------
static bool shape_count(int rank, const uint64_t* shape, uint64_t* count) {
    uint64_t c = 1;
    for (int i = 0; i < rank; i++) {
        if (shape[i] != 0 && c > UINT64_MAX / shape[i]) return false;
        c *= shape[i];
    }
    *count = c;
    return true;
}

mg_status buffer_new(Device* d, mg_dtype dtype, int rank, const uint64_t* shape, Buffer** out) {
    if (rank < 0 || rank > MG_MAX_RANK) return fail(MG_SHAPE_UNSUPPORTED, "rank %d is outside 0..%d", rank, MG_MAX_RANK);
    uint64_t count;
    if (!shape_count(rank, shape, &count) || count > (UINT64_MAX >> 3))
        return fail(MG_SHAPE_UNSUPPORTED, "buffer element count overflows");
    Buffer* b = new (std::nothrow) Buffer();
    if (!b) return fail(MG_EXECUTION_FAILED, "host allocation failed");
    b->device = d;
    b->dtype = dtype;
    b->rank = rank;
    for (int i = 0; i < rank; i++) b->shape[i] = shape[i];
    b->count = count;
    mg_status s = device_alloc(d, count * dtype_size(dtype), &b->ptr);
    if (s != MG_OK) {
        delete b;
        return s;
    }
    device_ref(d);
    *out = b;
    return MG_OK;
}

void buffer_drop_prep(Buffer* b) {
    if (b->prep || b->compact) b->device->prep_gen.fetch_add(1);
    if (b->prep) device_free(b->device, b->prep);
    b->prep = nullptr;
    b->prep_n = b->prep_k = b->prep_kp = 0;
    b->prep_transposed = -1;
    b->prep_one_term = false;
    if (b->compact) device_free(b->device, b->compact);
    b->compact = nullptr;
    b->compact_state = 0;
}

void buffer_free(Buffer* b) {
    if (!b) return;
    Device* d = b->device;
    buffer_drop_prep(b);
    if (b->owned && b->ptr) device_free(d, b->ptr);
    if (b->q8_scales) device_free(d, b->q8_scales);
    delete b;
    device_unref(d);
}

mg_status output_for(Device* d, mg_dtype dtype, int rank, const uint64_t* shape, mg_buffer** out,
                     Buffer** result) {
    if (!out) return fail(MG_INVALID_ARGUMENT, "null output parameter");
    uint64_t count;
    if (!shape_count(rank, shape, &count)) return fail(MG_SHAPE_UNSUPPORTED, "output element count overflows");
    Buffer* o = buf(*out);
    if (o && o->device == d && o->dtype == dtype && o->count == count) {
        buffer_drop_prep(o);  // its contents are about to change
        o->is_weight = false;
        o->rank = rank;
        for (int i = 0; i < rank; i++) o->shape[i] = shape[i];
        *result = o;
        return MG_OK;
    }
    Buffer* n = nullptr;
    MG_TRY(buffer_new(d, dtype, rank, shape, &n));
    *out = reinterpret_cast<mg_buffer*>(n);
    *result = n;
    return MG_OK;
}

void device_ref(Device* d) { d->refs.fetch_add(1); }

void device_unref(Device* d) {
    if (d->refs.fetch_sub(1) != 1) return;
    cudaSetDevice(d->ordinal);
    cudaStreamSynchronize(d->own_stream);  // the device's stream since mg_device_close
    for (void* p : d->held_frees) {  // parked for steps that are gone with their executors
        if (d->plain_allocs.erase(p)) cudaFree(p);
        else cudaFreeAsync(p, d->own_stream);
    }
    d->held_frees.clear();
    cudaStreamSynchronize(d->own_stream);
    cudaFree(d->flags);
    cudaFree(d->counters);
    cudaFreeHost(d->host_flags);
    cudaMemPoolDestroy(d->pool);
    cudaStreamDestroy(d->own_stream);
    delete d;
}

}  // namespace mg

using namespace mg;

// =========================================================================================
// C ABI: library, devices, buffers
// =========================================================================================
extern "C" {

int mg_abi_version(void) { return MG_ABI_VERSION; }

const char* mg_last_error(void) { return t_last_error.c_str(); }

const char* mg_status_name(mg_status s) {
    switch (s) {
        case MG_OK: return "Ok";
        case MG_SHAPE_UNSUPPORTED: return "ShapeUnsupported";
        case MG_DTYPE_UNSUPPORTED: return "DTypeUnsupported";
        case MG_LAYOUT_UNSUPPORTED: return "LayoutUnsupported";
        case MG_EXECUTION_FAILED: return "ExecutionFailed";
        case MG_OUT_OF_DEVICE_MEMORY: return "OutOfDeviceMemory";
        case MG_COMPILATION_FAILED: return "CompilationFailed";
        case MG_DRIVER_FAILED: return "DriverFailed";
        case MG_DEVICE_UNAVAILABLE: return "DeviceUnavailable";
        case MG_CAPTURE_UNSUPPORTED: return "CaptureUnsupported";
        case MG_KERNEL_NOT_FOUND: return "KernelNotFound";
        case MG_ATTRIBUTE_UNSUPPORTED: return "KernelAttributeUnsupported";
        case MG_INVALID_ARGUMENT: return "InvalidArgument";
        case MG_KERNEL_TIMEOUT: return "KernelTimeout";
    }
    return "Unknown";
}

mg_status mg_device_count(int* count) {
    if (!count) return fail(MG_INVALID_ARGUMENT, "null count");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;  // no driver or no device: zero devices, not an error
    }
    *count = n;
    return MG_OK;
}

mg_status mg_device_open(int ordinal, mg_device** out) {
    if (!out) return fail(MG_INVALID_ARGUMENT, "null output parameter");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || ordinal < 0 || ordinal >= n) {
        cudaGetLastError();
        return fail(MG_DEVICE_UNAVAILABLE, "no CUDA device cuda:%d (%d visible)", ordinal, n);
    }
    MG_CUDA(cudaSetDevice(ordinal), "selecting the device");
    cudaDeviceProp prop;
    MG_CUDA(cudaGetDeviceProperties(&prop, ordinal), "reading device properties");
    if (prop.major != 10)
        return fail(MG_DEVICE_UNAVAILABLE, "cuda:%d is sm_%d%d; this provider is built for sm_100a only",
                    ordinal, prop.major, prop.minor);
    Device* d = new (std::nothrow) Device();
    if (!d) return fail(MG_EXECUTION_FAILED, "host allocation failed");
    d->ordinal = ordinal;
    d->sm_count = prop.multiProcessorCount;
    d->sm_major = prop.major;
    d->sm_minor = prop.minor;
    const char* pdl = getenv("MAGNETAR_CUDA_PDL");
    d->pdl = !(pdl && pdl[0] == '0');
    cudaError_t e = cudaStreamCreateWithFlags(&d->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete d;
        return from_cuda(e, "creating the device stream");
    }
    d->stream = d->own_stream;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = ordinal;
    e = cudaMemPoolCreate(&d->pool, &props);
    if (e != cudaSuccess) {
        cudaStreamDestroy(d->own_stream);
        delete d;
        return from_cuda(e, "creating the memory pool");
    }
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(d->pool, cudaMemPoolAttrReleaseThreshold, &keep);
    e = cudaMalloc(&d->flags, 128);
    if (e == cudaSuccess) e = cudaMemset(d->flags, 0, 128);
    if (e == cudaSuccess) e = cudaMalloc(&d->counters, (1u << 16) * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(d->counters, 0, (1u << 16) * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMallocHost(&d->host_flags, 64);
    // The step offset shares the status words' allocation (bytes 32..39; the words use 0..15).
    d->step_offset = reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(d->flags) + 32);
    if (e != cudaSuccess) {
        if (d->flags) cudaFree(d->flags);
        if (d->counters) cudaFree(d->counters);
        cudaMemPoolDestroy(d->pool);
        cudaStreamDestroy(d->own_stream);
        delete d;
        return from_cuda(e, "allocating the status words");
    }
    *out = reinterpret_cast<mg_device*>(d);
    return MG_OK;
}

mg_status mg_device_close(mg_device* h) {
    if (!h) return MG_OK;
    Device* d = dev(h);
    if (d->closed.exchange(true)) return MG_OK;
    cudaSetDevice(d->ordinal);
    d->capturing = false;
    flush_deferred_frees(d);
    scratch_release(d);
    cudaStreamSynchronize(d->stream);
    // A stream the caller bound (mg_device_set_stream) may be destroyed once the handle is
    // closed: buffers released later free on the device's own stream.
    d->stream = d->own_stream;
    device_unref(d);  // the handle's reference: the device goes with its last buffer
    return MG_OK;
}

mg_status mg_device_get_info(mg_device* h, mg_device_info* info) {
    MG_TRY(device_check(h));
    if (!info) return fail(MG_INVALID_ARGUMENT, "null info");
    Device* d = dev(h);
    cudaDeviceProp prop;
    MG_CUDA(cudaGetDeviceProperties(&prop, d->ordinal), "reading device properties");
    memset(info, 0, sizeof *info);
    info->ordinal = d->ordinal;
    snprintf(info->name, sizeof info->name, "%s", prop.name);
    info->sm_major = prop.major;
    info->sm_minor = prop.minor;
    info->sm_count = prop.multiProcessorCount;
    size_t fr = 0, tot = 0;
    MG_CUDA(cudaMemGetInfo(&fr, &tot), "reading device memory");
    info->total_bytes = tot;
    info->free_bytes = fr;
    return MG_OK;
}

mg_status mg_device_synchronize(mg_device* h) {
    MG_TRY(device_check(h));
    MG_CUDA(cudaStreamSynchronize(dev(h)->stream), "synchronizing the device stream");
    return MG_OK;
}

void* mg_device_stream(mg_device* h) { return h ? (void*)dev(h)->stream : nullptr; }

mg_status mg_device_set_stream(mg_device* h, void* stream) {
    if (!h) return fail(MG_INVALID_ARGUMENT, "null device handle");
    dev(h)->stream = stream ? (cudaStream_t)stream : dev(h)->own_stream;
    return MG_OK;
}

mg_status mg_device_counters(mg_device* h, uint64_t* uploads, uint64_t* downloads) {
    if (!h) return fail(MG_INVALID_ARGUMENT, "null device handle");
    if (uploads) *uploads = dev(h)->uploads.load();
    if (downloads) *downloads = dev(h)->downloads.load();
    return MG_OK;
}

uint64_t mg_device_launch_count(mg_device* h) { return h ? dev(h)->launches.load() : 0; }

mg_status mg_buffer_create(mg_device* h, mg_dtype dtype, int rank, const uint64_t* shape, mg_buffer** out) {
    MG_TRY(device_check(h));
    if (!out || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (dtype != MG_F32 && dtype != MG_F16 && dtype != MG_BF16) return fail(MG_DTYPE_UNSUPPORTED, "unknown dtype %d", (int)dtype);
    Buffer* b = nullptr;
    MG_TRY(buffer_new(dev(h), dtype, rank, shape, &b));
    *out = reinterpret_cast<mg_buffer*>(b);
    return MG_OK;
}

mg_status mg_buffer_zeros(mg_device* h, mg_dtype dtype, int rank, const uint64_t* shape, mg_buffer** out) {
    MG_TRY(mg_buffer_create(h, dtype, rank, shape, out));
    Buffer* b = buf(*out);
    mg_status s = k::fill_zero(dev(h), b->ptr, b->count * dtype_size(dtype));
    if (s != MG_OK) {
        buffer_free(b);
        *out = nullptr;
    }
    return s;
}

mg_status mg_buffer_wrap(mg_device* h, mg_dtype dtype, int rank, const uint64_t* shape, void* ptr, mg_buffer** out) {
    if (!h || !out || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    MG_TRY(device_check(h));
    if (rank < 0 || rank > MG_MAX_RANK) return fail(MG_SHAPE_UNSUPPORTED, "rank %d is outside 0..%d", rank, MG_MAX_RANK);
    uint64_t count;
    if (!shape_count(rank, shape, &count)) return fail(MG_SHAPE_UNSUPPORTED, "element count overflows");
    Buffer* b = new (std::nothrow) Buffer();
    if (!b) return fail(MG_EXECUTION_FAILED, "host allocation failed");
    b->device = dev(h);
    b->dtype = dtype;
    b->rank = rank;
    for (int i = 0; i < rank; i++) b->shape[i] = shape[i];
    b->count = count;
    b->ptr = ptr;
    b->owned = false;
    device_ref(b->device);
    *out = reinterpret_cast<mg_buffer*>(b);
    return MG_OK;
}

mg_status mg_buffer_release(mg_buffer* h) {
    if (!h) return MG_OK;
    Buffer* b = buf(h);
    cudaSetDevice(b->device->ordinal);
    buffer_free(b);
    return MG_OK;
}

mg_status mg_buffer_upload(mg_buffer* h, const void* host, uint64_t bytes) {
    if (!h || (!host && bytes)) return fail(MG_INVALID_ARGUMENT, "null argument");
    Buffer* b = buf(h);
    if (b->dtype == MG_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "a packed weight is written by mg_buffer_upload_q8_0 only");
    if (bytes != b->count * dtype_size(b->dtype))
        return fail(MG_SHAPE_UNSUPPORTED, "%llu bytes cannot fill a %s buffer of shape %s",
                    (unsigned long long)bytes, dtype_name(b->dtype), shape_str(b).c_str());
    MG_CUDA(cudaSetDevice(b->device->ordinal), "selecting the device");
    buffer_drop_prep(b);
    if (bytes) MG_CUDA(cudaMemcpyAsync(b->ptr, host, bytes, cudaMemcpyHostToDevice, b->device->stream), "uploading");
    b->device->uploads.fetch_add(1);
    return MG_OK;
}

mg_status mg_buffer_download(const mg_buffer* h, void* host, uint64_t bytes) {
    if (!h || (!host && bytes)) return fail(MG_INVALID_ARGUMENT, "null argument");
    const Buffer* b = buf(h);
    if (b->dtype == MG_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "a packed weight downloads as f32 values only");
    if (bytes != b->count * dtype_size(b->dtype))
        return fail(MG_SHAPE_UNSUPPORTED, "%llu bytes cannot hold a %s buffer of shape %s",
                    (unsigned long long)bytes, dtype_name(b->dtype), shape_str(b).c_str());
    MG_CUDA(cudaSetDevice(b->device->ordinal), "selecting the device");
    if (bytes) MG_CUDA(cudaMemcpyAsync(host, b->ptr, bytes, cudaMemcpyDeviceToHost, b->device->stream), "downloading");
    MG_CUDA(cudaStreamSynchronize(b->device->stream), "waiting for the download");
    b->device->downloads.fetch_add(1);
    return MG_OK;
}

mg_status mg_buffer_upload_f32(mg_buffer* h, const float* host, uint64_t count) {
    if (!h || (!host && count)) return fail(MG_INVALID_ARGUMENT, "null argument");
    Buffer* b = buf(h);
    if (b->dtype == MG_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "a packed weight is written by mg_buffer_upload_q8_0 only");
    if (count != b->count)
        return fail(MG_SHAPE_UNSUPPORTED, "%llu values cannot fill a buffer of shape %s",
                    (unsigned long long)count, shape_str(b).c_str());
    if (b->dtype == MG_F32) return mg_buffer_upload(h, host, count * 4);
    Device* d = b->device;
    MG_CUDA(cudaSetDevice(d->ordinal), "selecting the device");
    void* staging = nullptr;
    MG_TRY(device_alloc(d, count * 4, &staging));
    cudaError_t e = cudaMemcpyAsync(staging, host, count * 4, cudaMemcpyHostToDevice, d->stream);
    mg_status s = e == cudaSuccess ? MG_OK : from_cuda(e, "uploading");
    if (s == MG_OK) s = k::encode_half(d, (const float*)staging, (uint16_t*)b->ptr, count, b->dtype);
    device_free(d, staging);
    if (s == MG_OK) d->uploads.fetch_add(1);
    return s;
}

mg_status mg_buffer_download_f32(const mg_buffer* h, float* host, uint64_t count) {
    if (!h || (!host && count)) return fail(MG_INVALID_ARGUMENT, "null argument");
    const Buffer* b = buf(h);
    if (count != b->count)
        return fail(MG_SHAPE_UNSUPPORTED, "%llu values cannot hold a buffer of shape %s",
                    (unsigned long long)count, shape_str(b).c_str());
    if (b->dtype == MG_F32) return mg_buffer_download(h, host, count * 4);
    Device* d = b->device;
    MG_CUDA(cudaSetDevice(d->ordinal), "selecting the device");
    void* staging = nullptr;
    MG_TRY(device_alloc(d, count * 4, &staging));
    mg_status s = b->dtype == MG_Q8_0 ? k::q8_dequantize(d, b, (float*)staging, false)
                                      : k::decode_half(d, (const uint16_t*)b->ptr, (float*)staging, count, b->dtype);
    if (s == MG_OK) {
        cudaError_t e = cudaMemcpyAsync(host, staging, count * 4, cudaMemcpyDeviceToHost, d->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
        if (e != cudaSuccess) s = from_cuda(e, "downloading");
    }
    device_free(d, staging);
    if (s == MG_OK) d->downloads.fetch_add(1);
    return s;
}

mg_status mg_buffer_download_rows(const mg_buffer* h, uint64_t first_row, uint64_t rows, float* host,
                                  uint64_t count) {
    if (!h || (!host && count)) return fail(MG_INVALID_ARGUMENT, "null argument");
    const Buffer* b = buf(h);
    if (b->rank != 2 || b->dtype != MG_F32)
        return fail(MG_SHAPE_UNSUPPORTED, "row reads need a rank-2 f32 buffer, got %s %s", dtype_name(b->dtype),
                    shape_str(b).c_str());
    uint64_t cols = b->shape[1];
    if (first_row > b->shape[0] || rows > b->shape[0] - first_row || count != rows * cols)
        return fail(MG_SHAPE_UNSUPPORTED, "rows [%llu, %llu) of %s do not fit %llu values",
                    (unsigned long long)first_row, (unsigned long long)(first_row + rows), shape_str(b).c_str(),
                    (unsigned long long)count);
    MG_CUDA(cudaSetDevice(b->device->ordinal), "selecting the device");
    if (count)
        MG_CUDA(cudaMemcpyAsync(host, (const float*)b->ptr + first_row * cols, count * 4, cudaMemcpyDeviceToHost,
                                b->device->stream),
                "downloading rows");
    MG_CUDA(cudaStreamSynchronize(b->device->stream), "waiting for the download");
    b->device->downloads.fetch_add(1);
    return MG_OK;
}

mg_status mg_buffer_shape(const mg_buffer* h, int* rank, uint64_t* shape) {
    if (!h || !rank) return fail(MG_INVALID_ARGUMENT, "null argument");
    const Buffer* b = buf(h);
    *rank = b->rank;
    if (shape)
        for (int i = 0; i < b->rank; i++) shape[i] = b->shape[i];
    return MG_OK;
}

mg_status mg_buffer_dtype(const mg_buffer* h, mg_dtype* dtype) {
    if (!h || !dtype) return fail(MG_INVALID_ARGUMENT, "null argument");
    *dtype = buf(h)->dtype;
    return MG_OK;
}

mg_status mg_buffer_reshape(mg_buffer* h, int rank, const uint64_t* shape) {
    if (!h || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (rank < 0 || rank > MG_MAX_RANK) return fail(MG_SHAPE_UNSUPPORTED, "rank %d is outside 0..%d", rank, MG_MAX_RANK);
    Buffer* b = buf(h);
    if (b->dtype == MG_Q8_0) return fail(MG_LAYOUT_UNSUPPORTED, "a packed weight keeps its logical shape");
    uint64_t count;
    if (!shape_count(rank, shape, &count) || count != b->count)
        return fail(MG_SHAPE_UNSUPPORTED, "cannot reshape %s to a different element count", shape_str(b).c_str());
    b->rank = rank;
    for (int i = 0; i < rank; i++) b->shape[i] = shape[i];
    return MG_OK;
}

void* mg_buffer_device_ptr(const mg_buffer* h) { return h ? buf(h)->ptr : nullptr; }

int mg_buffer_is_compact(const mg_buffer* h) {
    return h && (buf(h)->compact_state == 1 || buf(h)->dtype == MG_Q8_0) ? 1 : 0;
}

int mg_buffer_is_q8(const mg_buffer* h) { return h && buf(h)->dtype == MG_Q8_0 ? 1 : 0; }

// src/kernels.rs:1725-1838 (the Q8_0 branch): the blocks uploaded as they are and split on the
// device into quants and f32 scales.
mg_status mg_buffer_upload_q8_0(mg_device* h, const void* blocks, uint64_t bytes, uint64_t stored_rows,
                                uint64_t stored_cols, int transposed, mg_buffer** out) {
    MG_TRY(device_check(h));
    if (!out || (!blocks && bytes)) return fail(MG_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    Device* d = dev(h);
    if (stored_rows == 0 || stored_cols == 0 || stored_cols % 32 != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "a Q8_0 weight needs rows and a multiple of 32 columns, got [%llu, %llu]",
                    (unsigned long long)stored_rows, (unsigned long long)stored_cols);
    if (stored_rows > (UINT64_MAX >> 8) / stored_cols)
        return fail(MG_SHAPE_UNSUPPORTED, "Q8_0 weight element count overflows");
    const uint64_t nblocks = stored_rows * stored_cols / 32;
    if (bytes != nblocks * 34)
        return fail(MG_SHAPE_UNSUPPORTED, "%llu bytes are not the %llu blocks of a [%llu, %llu] Q8_0 weight",
                    (unsigned long long)bytes, (unsigned long long)nblocks, (unsigned long long)stored_rows,
                    (unsigned long long)stored_cols);
    if (d->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "a host-to-device upload cannot be captured");
    MG_CUDA(cudaSetDevice(d->ordinal), "selecting the device");
    const uint64_t shape[2] = {transposed ? stored_cols : stored_rows, transposed ? stored_rows : stored_cols};
    Buffer* b = nullptr;
    MG_TRY(buffer_new(d, MG_Q8_0, 2, shape, &b));
    b->q8_rows = stored_rows;
    b->q8_cols = stored_cols;
    b->q8_transposed = transposed ? 1 : 0;
    b->q8_tiled = transposed && stored_cols % 128 == 0 ? 1 : 0;
    void* staging = nullptr;
    mg_status s = MG_OK;
    if (b->q8_tiled) {  // padded: the allocation buffer_new made is too small
        device_free(d, b->ptr);
        b->ptr = nullptr;
        s = device_alloc(d, q8_quant_bytes(b), &b->ptr);
        if (s == MG_OK) s = k::fill_zero(d, b->ptr, q8_quant_bytes(b));
    }
    if (s == MG_OK) s = device_alloc(d, q8_scale_bytes(b), (void**)&b->q8_scales);
    if (s == MG_OK && b->q8_tiled) s = k::fill_zero(d, b->q8_scales, q8_scale_bytes(b));
    if (s == MG_OK) s = device_alloc(d, bytes, &staging);
    if (s == MG_OK) {
        cudaError_t e = cudaMemcpyAsync(staging, blocks, bytes, cudaMemcpyHostToDevice, d->stream);
        s = e == cudaSuccess ? MG_OK : from_cuda(e, "uploading");
    }
    if (s == MG_OK) s = k::q8_unpack(d, (const uint8_t*)staging, b);
    if (staging) device_free(d, staging);
    // Settled before it returns: the packed few-row matmul starts loading a packed weight before
    // its dependency wait, so no kernel that writes one may still be running then.
    if (s == MG_OK) {
        cudaError_t e = cudaStreamSynchronize(d->stream);
        if (e != cudaSuccess) s = from_cuda(e, "waiting for the packed weight");
    }
    if (s != MG_OK) {
        buffer_free(b);
        return s;
    }
    d->uploads.fetch_add(1);
    *out = reinterpret_cast<mg_buffer*>(b);
    return MG_OK;
}

mg_status mg_buffer_set_weight(mg_buffer* h, int is_weight) {
    if (!h) return fail(MG_INVALID_ARGUMENT, "null buffer");
    Buffer* b = buf(h);
    if (!is_weight) {
        cudaSetDevice(b->device->ordinal);
        buffer_drop_prep(b);
    }
    if (is_weight && !b->is_weight) b->weight_fresh = true;
    b->is_weight = is_weight != 0;
    return MG_OK;
}

}  // extern "C"
