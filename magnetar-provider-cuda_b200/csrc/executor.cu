// The executor behind the C ABI: ProviderExecutionApi over a device tensor table keyed by
// resource id.  Mirrors `CudaExecutor` (src/executor.rs:91-118, 1191-1321, 1422-2027):
//
//  - write_tensor / write_weight_tensor upload a HostTensor and replace the id's buffer;
//  - submit_kernel dispatches by kernel name, parsing the attributes the reference parses
//    with the same defaults and refusals, runs on the device stream, and stores the output
//    under the invocation's output id, offering that id's previous buffer for reuse (the
//    output-offer rule, src/executor.rs:1276-1321); a failed dispatch leaves the id's
//    previous value in place;
//  - step capture records the invocations into one CUDA graph and replays it, checking the
//    embedding-id flag after each replay (src/executor.rs:177-376, src/kernels.rs:1022-1350);
//  - with a tensor-parallel plan, weights keep this rank's share and every invocation that
//    reads a row-split weight is summed across ranks (src/multi/tensor_parallel.rs:440-539).
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "internal.h"

namespace mg {
mg_status comm_all_reduce_buffer(mg_comm* comm, Buffer* b);
int comm_rank(mg_comm* comm);
int comm_world(mg_comm* comm);
}  // namespace mg

using namespace mg;

// One captured step (src/executor.rs:177-376 `CapturedExecutorStep`): its graph, what a replay
// needs to know, and what the capture recorded so that a replay can tell whether the step's
// storage is still in place.
struct CapturedStep {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool has_embedding = false;
    bool advancing = false;
    uint64_t max_offset = UINT64_MAX;
    uint64_t kernels = 0;  // kernels one replay launches
    // Device blocks the graph addresses: none of them is freed while the step lives.
    std::vector<void*> blocks;
    // Every resource an invocation of the step read or wrote, as it was at capture time
    // (src/executor.rs record_captured_resources): the buffer and its device storage, and the
    // operand forms of a weight that a captured matmul reads instead of its values.
    struct Resource {
        Buffer* b;
        void* ptr;
        uint64_t count;
        void* prep;
        void* compact;
    };
    std::map<std::string, Resource> resources;
    // Embedding id resources and the vocabulary of their table (host-checked on replay writes).
    std::map<std::string, uint64_t> embedding_ids;
    uint64_t storage_gen = 0, prep_gen = 0;  // when the recorded state was last known current
    // Replays with host I/O whose host memory is pinned run as one graph launch: the input
    // copies, the replay offset, the step's own nodes (cloned), the output copies and the
    // embedding-flag read and reset, built once per distinct set of host buffers and kept here.
    struct IoGraph {
        std::vector<mg_step_io> io;  // the host side (ids point into `names`)
        std::vector<std::string> names;
        std::vector<void*> device;   // the device buffer each entry copies to or from
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        uint64_t* offset_word = nullptr;  // pinned host word holding the replay's offset
    };
    std::vector<IoGraph*> io_graphs;
    bool io_graph_failed = false;  // building one failed once: use separate copies from then on
};

// One entry of the executor's observation log (src/executor.rs:1082-1100, KernelObservation).
struct Observation {
    int kind;
    std::string kernel;
    uint64_t invocation;
    mg_status status;
};

struct mg_executor {
    Device* device = nullptr;
    mg_device* handle = nullptr;
    std::map<std::string, Buffer*> storage;
    // Bumped whenever an id's buffer is replaced or released (a captured step re-checks its
    // resources only when this moved since it last checked).
    uint64_t storage_gen = 0;
    std::mutex lock;
    uint64_t started = 0, completed = 0, failed = 0;
    // Observation log: the most recent MG_OBSERVATION_LOG_CAPACITY entries, oldest first (the
    // oldest half is dropped once twice the capacity is held, as the reference's log does).
    std::vector<Observation> observations;
    uint64_t next_invocation = 0;
    // step capture
    bool capturing = false;
    bool capture_has_embedding = false;
    uint64_t launches_at_capture = 0;
    std::map<std::string, CapturedStep::Resource> capture_resources;
    std::map<std::string, uint64_t> capture_embedding_ids;
    // Captured steps by id (src/executor.rs StepCaptureId); `current` is the one the
    // single-step calls (mg_executor_replay_step, ...) replay: the last one
    // mg_executor_end_step_capture made.
    std::map<uint64_t, CapturedStep*> steps;
    uint64_t next_step = 1;
    uint64_t current = 0;
    // Step capture only: plain matmuls of one input (weights as B) waiting to launch as one
    // grouped projection, with the ropes of their outputs folded into its epilogue.  Nothing
    // runs during a capture, so deferring a launch changes only the recorded order, and every
    // invocation that is not folded in launches the group first.
    struct Deferred {
        k::GemmArgs g;
        Buffer* a;
        Buffer* out;
        Buffer* rope_out;
    };
    std::vector<Deferred> deferred;
    bool deferred_rope = false;
    k::RopeArgs rope{};
    // Step capture only: an embedding lookup waiting to see whether the next invocation is an
    // rmsnorm of its rows (then both launch as one kernel).  At most one of the two kinds of
    // deferred launch is pending at a time.
    bool embed_pending = false;
    k::EmbedArgs embed{};
    // Advancing attributes of the step being captured (src/kernels.rs:1019-1062): launches
    // whose attribute is named here read the replay's offset from the device and record the
    // largest offset they stay in bounds for; the captured step keeps the least of those.
    std::set<std::string> advancing;
    uint64_t capture_max_offset = UINT64_MAX;
    // tensor parallel
    mg_comm* comm = nullptr;
    std::map<std::string, int> plan;            // weight id -> 0 columns, 1 rows
    std::set<std::string> sharded;              // activations holding a column share
};

namespace {

struct Attrs {
    const mg_invocation* inv;
    const mg_attribute* find(const char* name) const {
        for (int i = 0; i < inv->attribute_count; i++)
            if (inv->attributes[i].name && strcmp(inv->attributes[i].name, name) == 0) return &inv->attributes[i];
        return nullptr;
    }
    // src/executor.rs:1176-1185: only a Boolean counts, anything else is the default.
    bool boolean(const char* name, bool dflt) const {
        const mg_attribute* a = find(name);
        return a && a->kind == MG_ATTR_BOOL ? a->int_value != 0 : dflt;
    }
    // src/executor.rs:1141-1150
    float flt(const char* name, float dflt) const {
        const mg_attribute* a = find(name);
        return a && a->kind == MG_ATTR_FLOAT ? (float)a->float_value : dflt;
    }
    // src/executor.rs:1153-1164: present and not a Float is refused.
    mg_status flt_opt(const char* name, bool* present, float* value) const {
        const mg_attribute* a = find(name);
        *present = false;
        if (!a) return MG_OK;
        if (a->kind != MG_ATTR_FLOAT) return fail(MG_ATTRIBUTE_UNSUPPORTED, "%s must be a float", name);
        *present = true;
        *value = (float)a->float_value;
        return MG_OK;
    }
    // src/executor.rs:1166-1174: a non-negative Integer, else absent.
    bool integer(const char* name, uint64_t* value) const {
        const mg_attribute* a = find(name);
        if (a && a->kind == MG_ATTR_INT && a->int_value >= 0) {
            *value = (uint64_t)a->int_value;
            return true;
        }
        return false;
    }
    const char* string(const char* name) const {
        const mg_attribute* a = find(name);
        return a && a->kind == MG_ATTR_STRING ? a->string_value : nullptr;
    }
};

mg_status store_replace(mg_executor* ex, const std::string& id, Buffer* b) {
    auto it = ex->storage.find(id);
    if (it != ex->storage.end() && it->second != b) buffer_free(it->second);
    if (it == ex->storage.end() || it->second != b) ex->storage_gen++;
    ex->storage[id] = b;
    return MG_OK;
}

void io_graph_destroy(CapturedStep::IoGraph* g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    if (g->offset_word) cudaFreeHost(g->offset_word);
    delete g;
}

void step_destroy(mg_executor* ex, CapturedStep* st) {
    if (!st) return;
    cudaSetDevice(ex->device->ordinal);
    for (CapturedStep::IoGraph* g : st->io_graphs) io_graph_destroy(g);
    if (st->exec) cudaGraphExecDestroy(st->exec);
    if (st->graph) cudaGraphDestroy(st->graph);
    graph_release(ex->device, st->blocks);
    delete st;
}

void observe(mg_executor* ex, int kind, const char* kernel, uint64_t invocation, mg_status status) {
    if (ex->observations.size() >= 2 * MG_OBSERVATION_LOG_CAPACITY)
        ex->observations.erase(ex->observations.begin(), ex->observations.begin() + MG_OBSERVATION_LOG_CAPACITY);
    ex->observations.push_back({kind, kernel ? kernel : "", invocation, status});
}

// While capturing: records the device blocks and the storage of resource `id` (buffer `b`) for
// the step being captured.
void capture_record(mg_executor* ex, const std::string& id, Buffer* b) {
    if (!b) return;
    Device* d = ex->device;
    graph_touch(d, b->ptr);
    graph_touch(d, b->prep);
    graph_touch(d, b->compact);
    graph_touch(d, b->q8_scales);
    ex->capture_resources[id] = {b, b->ptr, b->count, b->prep, b->compact};
}

mg_status get_input(mg_executor* ex, const mg_invocation* inv, int index, Buffer** out) {
    if (index >= inv->input_count || !inv->inputs || !inv->inputs[index])
        return fail(MG_EXECUTION_FAILED, "missing input at index %d", index);
    auto it = ex->storage.find(inv->inputs[index]);
    if (it == ex->storage.end())
        return fail(MG_EXECUTION_FAILED, "no materialized data for input resource %s", inv->inputs[index]);
    *out = it->second;
    return MG_OK;
}

// While a step capture records: the device address of the replay offset for a launch whose
// `attribute` advances, after recording that the launch stays within bounds for offsets up to
// `max_offset` (src/kernels.rs:1425-1435).  Null outside a capture or for an attribute that
// does not advance.
const uint64_t* advancing_offset(mg_executor* ex, const char* attribute, uint64_t max_offset) {
    if (!ex->capturing || !ex->advancing.count(attribute)) return nullptr;
    ex->capture_max_offset = std::min(ex->capture_max_offset, max_offset);
    return ex->device->step_offset;
}

// src/executor.rs:1238-1249: accumulation_dtype, when given, must be f32.
mg_status require_f32_accumulation(const Attrs& at) {
    const char* s = at.string("accumulation_dtype");
    if (s && strcmp(s, "f32") != 0 && strcmp(s, "float32") != 0 && strcmp(s, "Float32") != 0)
        return fail(MG_DTYPE_UNSUPPORTED, "the CUDA Provider only accumulates in f32; requested %s", s);
    return MG_OK;
}

// YaRN's correction range (the published algorithm: the dimension index whose wavelength
// completes `rotations` turns over the original context), clamped to [0, dimension - 1].
void yarn_correction_range(double beta_fast, double beta_slow, uint64_t dimension, double base, double original,
                           float* low, float* high) {
    auto corr = [&](double rotations) {
        return (double)dimension * std::log(original / (rotations * 2.0 * M_PI)) / (2.0 * std::log(base));
    };
    double lo = std::floor(corr(beta_fast)), hi = std::ceil(corr(beta_slow));
    lo = lo < 0 ? 0 : lo;
    hi = hi > (double)(dimension - 1) ? (double)(dimension - 1) : hi;
    *low = (float)lo;
    *high = (float)hi;
}

inline mg_buffer* H(Buffer* b) { return reinterpret_cast<mg_buffer*>(b); }

// The rope attributes the reference parses (src/executor.rs:1563-1666), with its defaults and
// refusals.
mg_status parse_rope(const Attrs& at, mg_rope_params* p) {
    memset(p, 0, sizeof *p);
    p->base = at.flt("base", 10000.0f);
    p->scale = at.flt("scale", 1.0f);
    if (!at.integer("dimension", &p->dimension)) return fail(MG_ATTRIBUTE_UNSUPPORTED, "dimension");
    const char* mode = at.string("position_mode");
    if (mode && strcmp(mode, "sequential") != 0)
        return fail(MG_ATTRIBUTE_UNSUPPORTED, "position_mode '%s' is not implemented", mode);
    const mg_attribute* po = at.find("position_offset");
    if (po) {
        if (po->kind != MG_ATTR_INT) return fail(MG_ATTRIBUTE_UNSUPPORTED, "position_offset must be an integer");
        if (po->int_value < 0)
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "position_offset %lld must not be negative", (long long)po->int_value);
        p->position_offset = (uint64_t)po->int_value;
    }
    if (!at.integer("head_count", &p->head_count)) p->head_count = 1;
    const mg_attribute* pr = at.find("rotation_pairing");
    p->pairing = 0;
    if (pr) {
        if (pr->kind != MG_ATTR_STRING) return fail(MG_ATTRIBUTE_UNSUPPORTED, "rotation_pairing must be a string");
        if (!strcmp(pr->string_value, "interleaved")) p->pairing = 0;
        else if (!strcmp(pr->string_value, "half_split")) p->pairing = 1;
        else return fail(MG_ATTRIBUTE_UNSUPPORTED, "rotation_pairing '%s' is not implemented", pr->string_value);
    }
    const char* fs = at.string("frequency_scaling");
    p->amplitude = 1.0f;
    if (fs && !strcmp(fs, "yarn")) {
        const float factor = at.flt("factor", 0.0f);
        const float original = at.flt("original_context_length", 0.0f);
        if (!(factor > 0.0f) || !(original > 0.0f))
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "yarn needs a positive factor and original_context_length");
        p->yarn_factor = factor;
        yarn_correction_range(at.flt("beta_fast", 32.0f), at.flt("beta_slow", 1.0f), p->dimension, p->base, original,
                              &p->yarn_low, &p->yarn_high);
        p->amplitude = at.flt("attention_factor", 1.0f);
    } else if (fs && !strcmp(fs, "banded")) {
        p->banded_factor = at.flt("factor", 0.0f);
        p->low_freq_factor = at.flt("low_freq_factor", 0.0f);
        p->high_freq_factor = at.flt("high_freq_factor", 0.0f);
        p->original_context_length = at.flt("original_context_length", 0.0f);
        if (!(p->banded_factor > 0.0f) || !(p->low_freq_factor > 0.0f) || !(p->high_freq_factor > p->low_freq_factor) ||
            !(p->original_context_length > 0.0f))
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "banded frequency scaling needs factor > 0, 0 < low < high and a context length");
    } else if (fs) {
        return fail(MG_ATTRIBUTE_UNSUPPORTED, "frequency_scaling '%s' is not implemented", fs);
    }
    p->rotated_pairs = UINT64_MAX;
    const mg_attribute* prf = at.find("partial_rotary_factor");
    if (prf) {
        if (prf->kind != MG_ATTR_FLOAT || !(prf->float_value > 0.0) || prf->float_value > 1.0)
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "partial_rotary_factor must be a float in (0, 1]");
        p->rotated_pairs = (uint64_t)std::floor(prf->float_value * (double)p->dimension / 2.0);
    }
    return MG_OK;
}


// The body of run_invocation_with_offer (src/executor.rs:1422-2027).  `out` holds the
// offered previous output buffer (or null) and receives the result.
// An rmsnorm invocation's inputs and attributes (src/executor.rs:1586-1640).
struct RmsInv {
    Buffer* x = nullptr;
    Buffer* w = nullptr;
    float eps = 1e-6f;
    uint64_t hc = 0, hd = 0;
};

mg_status parse_rmsnorm(mg_executor* ex, const mg_invocation* inv, RmsInv* r) {
    Attrs at{inv};
    MG_TRY(get_input(ex, inv, 0, &r->x));
    if (inv->input_count > 1) MG_TRY(get_input(ex, inv, 1, &r->w));
    const mg_attribute* ws = at.find("with_scale");
    if (ws && ws->kind == MG_ATTR_BOOL && (ws->int_value != 0) != (r->w != nullptr))
        return fail(MG_ATTRIBUTE_UNSUPPORTED, "rmsnorm with_scale %s contradicts its %d input(s)",
                    ws->int_value ? "true" : "false", inv->input_count);
    bool have_hc = false, have_hd = false;
    for (const char* key : {"head_count", "head_dimension"}) {
        const mg_attribute* h = at.find(key);
        if (!h) continue;
        if (h->kind != MG_ATTR_INT || h->int_value <= 0)
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "rmsnorm %s must be a positive integer", key);
        if (!strcmp(key, "head_count")) {
            r->hc = (uint64_t)h->int_value;
            have_hc = true;
        } else {
            r->hd = (uint64_t)h->int_value;
            have_hd = true;
        }
    }
    if (have_hc != have_hd) return fail(MG_ATTRIBUTE_UNSUPPORTED, "rmsnorm head_count and head_dimension go together");
    r->eps = at.flt("epsilon", 1e-6f);
    return MG_OK;
}

mg_status dispatch(mg_executor* ex, const mg_invocation* inv, mg_buffer** out) {
    const char* name = inv->kernel;
    Attrs at{inv};
    mg_device* dh = ex->handle;
    Buffer *a = nullptr, *b = nullptr, *c = nullptr;
    if (!strcmp(name, "matmul") || !strcmp(name, "matmul-bias") || !strcmp(name, "matmul-residual") ||
        !strcmp(name, "gated-matmul")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        const int ta = at.boolean("transpose_a", false), tb = at.boolean("transpose_b", false);
        MG_TRY(require_f32_accumulation(at));
        if (!strcmp(name, "matmul")) return mg_matmul(dh, H(a), H(b), ta, tb, out);
        MG_TRY(get_input(ex, inv, 2, &c));
        if (!strcmp(name, "matmul-bias")) return mg_matmul_bias(dh, H(a), H(b), H(c), ta, tb, out);
        if (!strcmp(name, "matmul-residual")) return mg_matmul_residual(dh, H(a), H(b), H(c), ta, tb, out);
        return mg_gated_matmul(dh, H(a), H(b), H(c), ta, tb, out);
    }
    if (!strcmp(name, "silu-mul")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        return mg_silu_mul(dh, H(a), H(b), out);
    }
    if (!strcmp(name, "kv-write")) {
        // src/executor.rs:1366-1420: in place when the output is the store (a KV history), else
        // into a copy of the store kept under the output; a failed write leaves the rows as
        // they were.
        uint64_t row_offset = 0;
        if (!at.integer("row_offset", &row_offset))
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "kv-write needs a non-negative integer row_offset");
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        k::KvWriteArgs kw;
        MG_TRY(kv_write_plan(dh, H(a), H(b), row_offset, &kw));
        // An advancing row_offset writes at row_offset + offset (src/kernels.rs:2306-2310).
        kw.step = advancing_offset(ex, "row_offset", kw.capacity - (kw.row_offset + kw.count));
        const bool in_place = !strcmp(inv->inputs[0], inv->output);
        Buffer* target = a;
        if (!in_place) {
            MG_TRY(buffer_new(ex->device, a->dtype, a->rank, a->shape, &target));
            cudaError_t e = cudaMemcpyAsync(target->ptr, a->ptr, a->count * dtype_size(a->dtype),
                                            cudaMemcpyDeviceToDevice, ex->device->stream);
            if (e != cudaSuccess) {
                buffer_free(target);
                return from_cuda(e, "copying the kv-write store");
            }
            kw.store = (float*)target->ptr;
        } else {
            // A captured matmul may read the store through its operand form, which an in-place
            // write inside the same step would leave stale.
            if (ex->capturing && (a->prep || a->compact))
                return fail(MG_CAPTURE_UNSUPPORTED, "an in-place kv-write into a weight read through its operand form cannot be captured");
            buffer_drop_prep(a);
        }
        const mg_status s = k::kv_write(ex->device, kw);
        if (s != MG_OK) {
            if (!in_place) buffer_free(target);
            return s;
        }
        *out = H(target);
        return MG_OK;
    }
    if (!strcmp(name, "embedding")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        bool has_scale;
        float scale = 1.0f;
        MG_TRY(at.flt_opt("scale", &has_scale, &scale));
        if (ex->capturing) ex->capture_has_embedding = true;
        return mg_embedding(dh, H(a), H(b), has_scale ? 1 : 0, scale, out);
    }
    if (!strcmp(name, "rmsnorm")) {
        RmsInv r;
        MG_TRY(parse_rmsnorm(ex, inv, &r));
        return mg_rmsnorm(dh, H(r.x), r.w ? H(r.w) : nullptr, r.eps, r.hc, r.hd, out);
    }
    if (!strcmp(name, "rope")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        mg_rope_params p;
        MG_TRY(parse_rope(at, &p));
        k::RopeArgs ra;
        MG_TRY(rope_plan(dh, H(a), &p, out, &ra));
        ra.step = advancing_offset(ex, "position_offset", UINT64_MAX);
        return k::rope(ex->device, (const float*)a->ptr, (float*)buf(*out)->ptr, ra);
    }
    if (!strcmp(name, "attention")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        MG_TRY(get_input(ex, inv, 2, &c));
        mg_attention_params p;
        memset(&p, 0, sizeof p);
        if (!at.integer("head_count", &p.head_count)) return fail(MG_ATTRIBUTE_UNSUPPORTED, "head_count");
        if (!at.integer("head_dimension", &p.head_dimension)) return fail(MG_ATTRIBUTE_UNSUPPORTED, "head_dimension");
        uint64_t v;
        p.kv_head_count = at.integer("kv_head_count", &v) ? v : 0;
        p.window_size = at.integer("window_size", &v) ? (int64_t)v : -1;
        p.causal = at.boolean("causal", false);
        const char* mk = at.string("attention_mask_kind");
        if (mk) {
            bool expected;
            if (!strcmp(mk, "causal")) expected = true;
            else if (!strcmp(mk, "bidirectional")) expected = false;
            else return fail(MG_ATTRIBUTE_UNSUPPORTED, "attention_mask_kind '%s' is not implemented", mk);
            if (expected != (p.causal != 0))
                return fail(MG_ATTRIBUTE_UNSUPPORTED, "attention_mask_kind '%s' is inconsistent with causal=%s", mk,
                            p.causal ? "true" : "false");
        }
        p.key_count = at.integer("key_count", &v) ? (int64_t)v : -1;
        bool has_scale;
        float scale = 0.0f;
        MG_TRY(at.flt_opt("scale", &has_scale, &scale));
        p.has_scale = has_scale;
        p.scale = scale;
        const mg_attribute* vd = at.find("value_head_dimension");
        if (vd) {
            if (vd->kind != MG_ATTR_INT || vd->int_value <= 0)
                return fail(MG_ATTRIBUTE_UNSUPPORTED, "value_head_dimension must be a positive integer");
            p.value_dimension = (uint64_t)vd->int_value;
        }
        if (at.find("value_head_stride") || at.find("latent_kv_width"))
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "latent and strided-value attention forms are not implemented");
        k::AttentionArgs aa;
        MG_TRY(attention_plan(dh, H(a), H(b), H(c), &p, out, &aa));
        // An advancing key_count admits key_count + offset keys (src/kernels.rs:6630-6640).
        if (p.key_count >= 0) aa.step = advancing_offset(ex, "key_count", aa.kv_rows - aa.kv_seq_len);
        return k::attention(ex->device, aa);
    }
    if (!strcmp(name, "softmax")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        return mg_softmax(dh, H(a), out);
    }
    if (!strcmp(name, "silu")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        return mg_silu(dh, H(a), out);
    }
    if (!strcmp(name, "gelu")) {
        // src/executor.rs:1817-1828: the tanh approximation, the only one implemented
        MG_TRY(get_input(ex, inv, 0, &a));
        const mg_attribute* ap = at.find("approximate");
        if (ap && !(ap->kind == MG_ATTR_STRING && ap->string_value && !strcmp(ap->string_value, "tanh")))
            return fail(MG_ATTRIBUTE_UNSUPPORTED, "gelu approximate %s is not implemented",
                        ap->kind == MG_ATTR_STRING && ap->string_value ? ap->string_value : "(not a string)");
        return mg_gelu_tanh(dh, H(a), out);
    }
    if (!strcmp(name, "row-scale")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        return mg_row_scale(dh, H(a), H(b), out);
    }
    if (!strcmp(name, "concat")) {
        // src/executor.rs:1933-1965: along the rows, or head by head (axis "heads"); a missing
        // axis concatenates rows
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        const mg_attribute* ax = at.find("axis");
        const char* axis = ax && ax->kind == MG_ATTR_STRING ? ax->string_value : nullptr;
        if (!ax || (axis && !strcmp(axis, "rows"))) return mg_concat(dh, H(a), H(b), out);
        if (axis && !strcmp(axis, "heads")) {
            uint64_t hc = 0, shc = 0;
            if (!at.integer("head_count", &hc)) return fail(MG_ATTRIBUTE_UNSUPPORTED, "head_count");
            if (!at.integer("second_head_count", &shc)) shc = hc;
            return mg_concat_heads(dh, H(a), H(b), hc, shc, out);
        }
        return fail(MG_ATTRIBUTE_UNSUPPORTED, "concat axis must be 'rows' or 'heads'");
    }
    if (!strcmp(name, "batched-matmul")) {
        // src/executor.rs:1798-1808
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        uint64_t groups = 0;
        if (!at.integer("group_count", &groups) || groups == 0) return fail(MG_ATTRIBUTE_UNSUPPORTED, "group_count");
        return mg_batched_matmul(dh, H(a), H(b), groups, at.boolean("transpose_b", false), out);
    }
    if (!strcmp(name, "activation")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        const char* kind = at.string("kind");
        if (kind && !strcmp(kind, "silu")) return mg_silu(dh, H(a), out);
        if (kind && !strcmp(kind, "scale")) {
            bool present;
            float f = 1.0f;
            MG_TRY(at.flt_opt("factor", &present, &f));
            if (!present) return fail(MG_ATTRIBUTE_UNSUPPORTED, "scale needs a factor");
            return mg_scale(dh, H(a), f, out);
        }
        // src/executor.rs:1829-1860
        if (kind && !strcmp(kind, "sigmoid")) return mg_sigmoid(dh, H(a), out);
        if (kind && !strcmp(kind, "softcap")) {
            bool present;
            float cap = 0.0f;
            MG_TRY(at.flt_opt("cap", &present, &cap));
            if (!present) return fail(MG_ATTRIBUTE_UNSUPPORTED, "softcap needs a cap");
            return mg_softcap(dh, H(a), cap, out);
        }
        return fail(MG_ATTRIBUTE_UNSUPPORTED, "activation kind %s is not implemented", kind ? kind : "(none)");
    }
    if (!strcmp(name, "add")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        return mg_add(dh, H(a), H(b), out);
    }
    if (!strcmp(name, "mul")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        return mg_mul(dh, H(a), H(b), out);
    }
    if (!strcmp(name, "residual-add")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        return mg_residual_add(dh, H(a), H(b), out);
    }
    if (!strcmp(name, "add-half") || !strcmp(name, "mul-half")) {
        MG_TRY(get_input(ex, inv, 0, &a));
        MG_TRY(get_input(ex, inv, 1, &b));
        // src/executor.rs:71-79: the first input's descriptor names the half dtype.
        const int dt = inv->input_dtypes ? inv->input_dtypes[0] : MG_F32;
        if (dt != MG_F16 && dt != MG_BF16)
            return fail(MG_DTYPE_UNSUPPORTED, "%s needs an f16 or bf16 input descriptor", name);
        const int op = !strcmp(name, "mul-half");
        if (a->dtype == MG_F32) return mg_half_binary_f32(dh, H(a), H(b), (mg_dtype)dt, op, out);
        return op ? mg_mul_half(dh, H(a), H(b), out) : mg_add_half(dh, H(a), H(b), out);
    }
    return fail(MG_KERNEL_NOT_FOUND, "kernel '%s' is not provided", name);
}

// ---- step-capture fusion ---------------------------------------------------------------------
// Launches what is deferred: the pending embedding lookup, or the deferred group -- one grouped
// projection (with its ropes), or a lone matmul.
mg_status flush_deferred(mg_executor* ex) {
    if (ex->embed_pending) {
        ex->embed_pending = false;
        const k::EmbedArgs& e = ex->embed;
        return k::embedding_run(ex->device, e, ex->device->flags);
    }
    if (ex->deferred.empty()) return MG_OK;
    k::GemmArgs gs[3];
    float* ro[3] = {nullptr, nullptr, nullptr};
    const int n = (int)ex->deferred.size();
    for (int i = 0; i < n; i++) {
        gs[i] = ex->deferred[i].g;
        ro[i] = ex->deferred[i].rope_out ? (float*)ex->deferred[i].rope_out->ptr : nullptr;
    }
    const bool rope = ex->deferred_rope;
    ex->deferred.clear();
    ex->deferred_rope = false;
    if (n == 1 && !rope) return k::gemm(ex->device, gs[0]);
    return k::gemm_group(ex->device, gs, n, rope ? &ex->rope : nullptr, ro);
}

bool deferred_uses(const mg_executor* ex, const Buffer* b) {
    for (const auto& d : ex->deferred)
        if (d.a == b || d.out == b || d.rope_out == b) return true;
    return false;
}

bool deferred_writes(const mg_executor* ex, const Buffer* b) {
    for (const auto& d : ex->deferred)
        if (d.out == b || d.rope_out == b) return true;
    return false;
}

bool same_rope(const k::RopeArgs& x, const k::RopeArgs& y) {
    return x.rows == y.rows && x.cols == y.cols && x.half == y.half && x.dimension == y.dimension &&
           x.position_offset == y.position_offset && x.head_count == y.head_count && x.rotated_pairs == y.rotated_pairs &&
           x.base == y.base && x.scale == y.scale && x.banded_factor == y.banded_factor &&
           x.low_freq_factor == y.low_freq_factor && x.high_freq_factor == y.high_freq_factor &&
           x.original_context_length == y.original_context_length && x.yarn_factor == y.yarn_factor &&
           x.yarn_low == y.yarn_low && x.yarn_high == y.yarn_high && x.amplitude == y.amplitude &&
           x.half_split == y.half_split && x.step == y.step;
}

// During a step capture: takes a plain matmul whose B is a weight into the deferred group (or
// starts a new group), or folds a rope of a deferred matmul's output into the group's
// epilogue.  Returns false when the invocation runs the ordinary way (the caller launches the
// group first); true when it was handled here, with its output in *result and its status in
// *status.  Validation and the output follow the ordinary call exactly (matmul_plan,
// rope_plan), so errors and the output-offer rule are unchanged.
bool capture_defer(mg_executor* ex, const mg_invocation* inv, mg_buffer* offered, mg_buffer** result,
                   mg_status* status) {
    Attrs at{inv};
    if (!strcmp(inv->kernel, "embedding")) {
        // Deferred until the next invocation shows whether an rmsnorm of its rows follows.
        Buffer *table = nullptr, *ids = nullptr;
        if (get_input(ex, inv, 0, &table) != MG_OK || get_input(ex, inv, 1, &ids) != MG_OK) return false;
        bool has_scale = false;
        float scale = 1.0f;
        if (at.flt_opt("scale", &has_scale, &scale) != MG_OK) return false;  // the ordinary call reports it
        *status = flush_deferred(ex);
        if (*status != MG_OK) return true;
        mg_buffer* res = offered;
        *status = embedding_plan(ex->handle, H(table), H(ids), has_scale ? 1 : 0, scale, &res, &ex->embed);
        *result = res;
        if (*status != MG_OK) return true;
        ex->embed_pending = true;
        ex->capture_has_embedding = true;
        return true;
    }
    if (ex->embed_pending && !strcmp(inv->kernel, "rmsnorm")) {
        RmsInv r;
        if (parse_rmsnorm(ex, inv, &r) != MG_OK || (float*)r.x->ptr != ex->embed.out) return false;
        if (offered && (float*)buf(offered)->ptr == ex->embed.out) return false;  // in place
        k::RmsArgs ra;
        mg_buffer* res = offered;
        *status = rmsnorm_plan(ex->handle, H(r.x), r.w ? H(r.w) : nullptr, r.eps, r.hc, r.hd, &res, &ra);
        *result = res;
        if (*status != MG_OK) return true;
        if (!k::embedding_rmsnorm_eligible(ex->embed, ra)) {
            *status = flush_deferred(ex);
            if (*status == MG_OK) *status = k::rmsnorm(ex->device, ra.x, ra.w, ra.out, ra.rows, ra.cols, ra.w_stride, ra.eps);
            return true;
        }
        ex->embed_pending = false;
        *status = k::embedding_rmsnorm(ex->device, ex->embed, ra, ex->device->flags);
        return true;
    }
    const bool is_mm = !strcmp(inv->kernel, "matmul"), is_rope = !strcmp(inv->kernel, "rope");
    if (!is_mm && !is_rope) return false;
    if (ex->embed_pending) {  // a matmul or rope after an embedding: the lookup launches first
        *status = flush_deferred(ex);
        if (*status != MG_OK) {
            *result = offered;
            return true;
        }
    }
    if (offered && deferred_uses(ex, buf(offered))) return false;
    Device* d = ex->device;
    if (is_mm) {
        Buffer *a = nullptr, *b = nullptr;
        if (get_input(ex, inv, 0, &a) != MG_OK || get_input(ex, inv, 1, &b) != MG_OK) return false;
        if (at.boolean("transpose_a", false) || at.boolean("transpose_b", false)) return false;
        if (require_f32_accumulation(at) != MG_OK || !b->is_weight) return false;
        if (deferred_writes(ex, a) || deferred_writes(ex, b)) return false;
        k::GemmArgs g;
        mg_buffer* res = offered;
        mg_status s = matmul_plan(ex->handle, H(a), H(b), nullptr, nullptr, 0, 0, 0, &res, &g);
        *result = res;
        if (s != MG_OK) {
            *status = s;
            return true;
        }
        const size_t n = ex->deferred.size();
        bool joined = false;
        if (n > 0 && n < 3 && ex->deferred[0].a == a && g.b_prep[0]) {
            k::GemmArgs gs[3];
            float* ro[3] = {nullptr, nullptr, nullptr};
            for (size_t i = 0; i < n; i++) {
                gs[i] = ex->deferred[i].g;
                ro[i] = ex->deferred[i].rope_out ? (float*)ex->deferred[i].rope_out->ptr : nullptr;
            }
            gs[n] = g;
            joined = k::gemm_group_eligible(gs, (int)n + 1, ex->deferred_rope ? &ex->rope : nullptr, ro);
        }
        if (!joined) {
            s = flush_deferred(ex);
            if (s == MG_OK && !(g.b_prep[0] && k::gemm_group_eligible(&g, 1, nullptr, nullptr))) {
                *status = k::gemm(d, g);  // not groupable: launched now
                return true;
            }
            if (s != MG_OK) {
                *status = s;
                return true;
            }
        }
        ex->deferred.push_back({g, a, buf(res), nullptr});
        *status = MG_OK;
        return true;
    }
    // a rope of a deferred matmul's output
    Buffer* x = nullptr;
    if (get_input(ex, inv, 0, &x) != MG_OK) return false;
    int member = -1;
    for (size_t i = 0; i < ex->deferred.size(); i++)
        if (ex->deferred[i].out == x && !ex->deferred[i].rope_out) member = (int)i;
    if (member < 0) return false;
    mg_rope_params rp;
    if (parse_rope(at, &rp) != MG_OK) return false;  // the ordinary call reports it
    k::RopeArgs ra;
    mg_buffer* res = offered;
    mg_status s = rope_plan(ex->handle, H(x), &rp, &res, &ra);
    *result = res;
    if (s != MG_OK) {
        *status = s;
        return true;
    }
    ra.step = advancing_offset(ex, "position_offset", UINT64_MAX);
    bool attach = !deferred_uses(ex, buf(res)) && (!ex->deferred_rope || same_rope(ex->rope, ra));
    if (attach) {
        const size_t n = ex->deferred.size();
        k::GemmArgs gs[3];
        float* ro[3] = {nullptr, nullptr, nullptr};
        for (size_t i = 0; i < n; i++) {
            gs[i] = ex->deferred[i].g;
            ro[i] = ex->deferred[i].rope_out ? (float*)ex->deferred[i].rope_out->ptr : nullptr;
        }
        ro[member] = (float*)buf(res)->ptr;
        attach = k::gemm_group_eligible(gs, (int)n, &ra, ro);
    }
    if (!attach) {  // the group launches, then this rope on its own
        s = flush_deferred(ex);
        *status = s == MG_OK ? k::rope(d, (const float*)x->ptr, (float*)buf(res)->ptr, ra) : s;
        return true;
    }
    ex->deferred[member].rope_out = buf(res);
    ex->rope = ra;
    ex->deferred_rope = true;
    *status = MG_OK;
    return true;
}

// Role of an invocation's output under the tensor-parallel plan
// (src/multi/tensor_parallel.rs:136-150): 2 partial (reads a row-split weight),
// 1 sharded (reads a column share), 0 replicated.
int tp_role(mg_executor* ex, const mg_invocation* inv) {
    int role = 0;
    for (int i = 0; i < inv->input_count; i++) {
        const std::string id = inv->inputs[i];
        auto it = ex->plan.find(id);
        if (it != ex->plan.end()) {
            if (it->second == 1) return 2;
            role = 1;
        } else if (ex->sharded.count(id)) {
            role = 1;
        }
    }
    return role;
}

mg_status upload_tensor(mg_executor* ex, const char* id, int rank, const uint64_t* shape, const float* data,
                        bool weight = false) {
    Buffer* nb = nullptr;
    MG_TRY(buffer_new(ex->device, MG_F32, rank, shape, &nb));
    nb->is_weight = weight;
    if (nb->count) {
        cudaError_t e = cudaMemcpyAsync(nb->ptr, data, nb->count * 4, cudaMemcpyHostToDevice, ex->device->stream);
        if (e != cudaSuccess) {
            buffer_free(nb);
            return from_cuda(e, "CUDA device upload failed");
        }
    }
    ex->device->uploads.fetch_add(1);
    store_replace(ex, id, nb);
    ex->sharded.erase(id);
    return MG_OK;
}

}  // namespace

namespace mg {
// [start, end) share of `extent` for `member` of `parts`, aligned to 32-element blocks when
// every part can hold one (src/multi/tensor_parallel.rs:82-86, 300-307).
void tp_share(uint64_t extent, int parts, int member, uint64_t* start, uint64_t* end) {
    const uint64_t granule = (extent % 32 == 0 && extent >= 32ull * (uint64_t)parts) ? 32 : 1;
    const uint64_t units = extent / granule;
    *start = units * (uint64_t)member / (uint64_t)parts * granule;
    *end = units * (uint64_t)(member + 1) / (uint64_t)parts * granule;
}
}  // namespace mg

extern "C" {

mg_status mg_tp_share(uint64_t extent, int parts, int member, uint64_t* start, uint64_t* end) {
    if (!start || !end) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (parts <= 0 || member < 0 || member >= parts) return fail(MG_SHAPE_UNSUPPORTED, "member %d of %d parts", member, parts);
    tp_share(extent, parts, member, start, end);
    return MG_OK;
}

mg_status mg_executor_create(mg_device* h, mg_executor** out) {
    MG_TRY(device_check(h));
    if (!out) return fail(MG_INVALID_ARGUMENT, "null output parameter");
    mg_executor* ex = new (std::nothrow) mg_executor();
    if (!ex) return fail(MG_EXECUTION_FAILED, "host allocation failed");
    ex->device = dev(h);
    ex->handle = h;
    device_ref(ex->device);  // its captured steps release device memory when it goes
    *out = ex;
    return MG_OK;
}

mg_status mg_executor_destroy(mg_executor* ex) {
    if (!ex) return MG_OK;
    cudaSetDevice(ex->device->ordinal);
    if (ex->capturing) mg_executor_abort_step_capture(ex);
    for (auto& kv : ex->steps) step_destroy(ex, kv.second);
    ex->steps.clear();
    for (auto& kv : ex->storage) buffer_free(kv.second);
    device_unref(ex->device);
    delete ex;
    return MG_OK;
}

mg_status mg_executor_write_tensor(mg_executor* ex, const char* id, int rank, const uint64_t* shape, const float* data) {
    if (!ex || !id || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    MG_TRY(device_check(ex->handle));
    return upload_tensor(ex, id, rank, shape, data);
}

// src/executor.rs:404-420: a packed weight stored as the checkpoint stored it.
mg_status mg_executor_write_packed_weight_tensor(mg_executor* ex, const char* id, int format, const void* blocks,
                                                 uint64_t bytes, uint64_t stored_rows, uint64_t stored_cols,
                                                 int transposed) {
    if (!ex || !id) return fail(MG_INVALID_ARGUMENT, "null argument");
    if (format != MG_PACKED_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "packed weight format %d is not supported", format);
    std::lock_guard<std::mutex> g(ex->lock);
    MG_TRY(device_check(ex->handle));
    if (ex->comm && ex->plan.count(id))
        return fail(MG_LAYOUT_UNSUPPORTED, "a packed weight cannot be split for tensor parallelism");
    mg_buffer* b = nullptr;
    MG_TRY(mg_buffer_upload_q8_0(ex->handle, blocks, bytes, stored_rows, stored_cols, transposed, &b));
    store_replace(ex, id, buf(b));
    ex->sharded.erase(id);
    return MG_OK;
}

mg_status mg_executor_write_weight_tensor(mg_executor* ex, const char* id, int rank, const uint64_t* shape,
                                          const float* data) {
    if (!ex || !id || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    MG_TRY(device_check(ex->handle));
    auto it = ex->plan.find(id);
    if (!ex->comm || it == ex->plan.end() || rank == 0) return upload_tensor(ex, id, rank, shape, data, true);
    // This rank's share (src/multi/tensor_parallel.rs:206-236).
    const int parts = comm_world(ex->comm), member = comm_rank(ex->comm);
    uint64_t local[MG_MAX_RANK];
    for (int i = 0; i < rank; i++) local[i] = shape[i];
    uint64_t count = 1;
    for (int i = 0; i < rank; i++) count *= shape[i];
    std::vector<float> part;
    if (it->second == 0) {  // columns: last dimension
        const uint64_t cols = shape[rank - 1], rows = cols ? count / cols : 0;
        uint64_t s, e;
        tp_share(cols, parts, member, &s, &e);
        local[rank - 1] = e - s;
        part.resize(rows * (e - s));
        for (uint64_t r = 0; r < rows; r++)
            memcpy(&part[r * (e - s)], data + r * cols + s, (e - s) * sizeof(float));
    } else {  // rows: first dimension
        const uint64_t rows = shape[0], per = rows ? count / rows : 0;
        uint64_t s, e;
        tp_share(rows, parts, member, &s, &e);
        local[0] = e - s;
        part.assign(data + s * per, data + e * per);
    }
    return upload_tensor(ex, id, rank, local, part.data(), true);
}

mg_status mg_executor_write_zeroed_tensor(mg_executor* ex, const char* id, int rank, const uint64_t* shape) {
    if (!ex || !id || (rank > 0 && !shape)) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    MG_TRY(device_check(ex->handle));
    Buffer* nb = nullptr;
    MG_TRY(buffer_new(ex->device, MG_F32, rank, shape, &nb));
    mg_status s = k::fill_zero(ex->device, nb->ptr, nb->count * 4);
    if (s != MG_OK) {
        buffer_free(nb);
        return s;
    }
    store_replace(ex, id, nb);
    ex->sharded.erase(id);
    return MG_OK;
}

mg_status mg_executor_adopt_buffer(mg_executor* ex, const char* id, mg_buffer* b) {
    if (!ex || !id || !b) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    if (buf(b)->device != ex->device) return fail(MG_INVALID_ARGUMENT, "buffer belongs to another device");
    store_replace(ex, id, buf(b));
    ex->sharded.erase(id);
    return MG_OK;
}

mg_status mg_executor_buffer(mg_executor* ex, const char* id, mg_buffer** out) {
    if (!ex || !id || !out) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    auto it = ex->storage.find(id);
    if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", id);
    *out = H(it->second);
    return MG_OK;
}

mg_status mg_executor_read_tensor(mg_executor* ex, const char* id, float* data, uint64_t capacity, int* rank,
                                  uint64_t* shape) {
    if (!ex || !id) return fail(MG_INVALID_ARGUMENT, "null argument");
    Buffer* b;
    {
        std::lock_guard<std::mutex> g(ex->lock);
        auto it = ex->storage.find(id);
        if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", id);
        b = it->second;
    }
    if (rank) *rank = b->rank;
    if (shape)
        for (int i = 0; i < b->rank; i++) shape[i] = b->shape[i];
    if (!data) return MG_OK;
    if (capacity < b->count)
        return fail(MG_SHAPE_UNSUPPORTED, "%llu values cannot hold resource %s of shape %s", (unsigned long long)capacity, id,
                    shape_str(b).c_str());
    return mg_buffer_download_f32(H(b), data, b->count);
}

// src/executor.rs:2549-2563: greedy selection over a resident logits tensor.
mg_status mg_executor_select_greedy_column(mg_executor* ex, const char* id, uint64_t row, const uint64_t* excluded,
                                           uint32_t excluded_count, float temperature, int* found, uint64_t* column) {
    if (!ex || !id || !found || !column) return fail(MG_INVALID_ARGUMENT, "null argument");
    *found = 0;
    Buffer* b;
    {
        std::lock_guard<std::mutex> g(ex->lock);
        auto it = ex->storage.find(id);
        if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", id);
        b = it->second;
    }
    return mg_greedy_select(ex->handle, H(b), row, excluded, excluded_count, temperature, found, column);
}

mg_status mg_executor_read_tensor_rows(mg_executor* ex, const char* id, uint64_t first_row, uint64_t rows, float* data,
                                       uint64_t capacity) {
    if (!ex || !id) return fail(MG_INVALID_ARGUMENT, "null argument");
    Buffer* b;
    {
        std::lock_guard<std::mutex> g(ex->lock);
        auto it = ex->storage.find(id);
        if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", id);
        b = it->second;
    }
    if (b->rank != 2) return fail(MG_SHAPE_UNSUPPORTED, "row reads need a rank-2 resource, got %s", shape_str(b).c_str());
    if (capacity < rows * b->shape[1]) return fail(MG_SHAPE_UNSUPPORTED, "row read does not fit %llu values", (unsigned long long)capacity);
    return mg_buffer_download_rows(H(b), first_row, rows, data, rows * b->shape[1]);
}

mg_status mg_executor_release_tensor(mg_executor* ex, const char* id, int* released) {
    if (!ex || !id) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    auto it = ex->storage.find(id);
    int r = 0;
    if (it != ex->storage.end()) {
        cudaSetDevice(ex->device->ordinal);
        buffer_free(it->second);
        ex->storage.erase(it);
        ex->storage_gen++;
        r = 1;
    }
    ex->plan.erase(id);
    ex->sharded.erase(id);
    if (released) *released = r;
    return MG_OK;
}

mg_status mg_executor_resident_shape(mg_executor* ex, const char* id, int* present, int* rank, uint64_t* shape) {
    if (!ex || !id || !present) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    auto it = ex->storage.find(id);
    *present = it != ex->storage.end();
    if (*present) {
        if (rank) *rank = it->second->rank;
        if (shape)
            for (int i = 0; i < it->second->rank; i++) shape[i] = it->second->shape[i];
    }
    return MG_OK;
}

mg_status mg_executor_copy_tensor(mg_executor* ex, const char* from, const char* to) {
    if (!ex || !from || !to) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    MG_TRY(device_check(ex->handle));
    auto it = ex->storage.find(from);
    if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", from);
    if (!strcmp(from, to)) return MG_OK;
    Buffer* src = it->second;
    Buffer* nb = nullptr;
    MG_TRY(buffer_new(ex->device, src->dtype, src->rank, src->shape, &nb));
    cudaError_t e = cudaSuccess;
    if (src->dtype == MG_Q8_0) {  // a packed weight: its layout, quants and scales
        nb->q8_rows = src->q8_rows;
        nb->q8_cols = src->q8_cols;
        nb->q8_transposed = src->q8_transposed;
        nb->q8_tiled = src->q8_tiled;
        device_free(ex->device, nb->ptr);
        nb->ptr = nullptr;
        mg_status s = device_alloc(ex->device, q8_quant_bytes(src), &nb->ptr);
        if (s == MG_OK) s = device_alloc(ex->device, q8_scale_bytes(src), (void**)&nb->q8_scales);
        if (s != MG_OK) {
            buffer_free(nb);
            return s;
        }
        e = cudaMemcpyAsync(nb->ptr, src->ptr, q8_quant_bytes(src), cudaMemcpyDeviceToDevice, ex->device->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(nb->q8_scales, src->q8_scales, q8_scale_bytes(src), cudaMemcpyDeviceToDevice,
                                ex->device->stream);
    } else {
        e = cudaMemcpyAsync(nb->ptr, src->ptr, src->count * dtype_size(src->dtype), cudaMemcpyDeviceToDevice,
                            ex->device->stream);
    }
    if (e != cudaSuccess) {
        buffer_free(nb);
        return from_cuda(e, "copying a resource");
    }
    store_replace(ex, to, nb);
    if (ex->sharded.count(from)) ex->sharded.insert(to);
    else ex->sharded.erase(to);
    return MG_OK;
}

mg_status mg_executor_submit_kernel(mg_executor* ex, const mg_invocation* inv) {
    if (!ex || !inv || !inv->kernel || !inv->output) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    ex->started++;
    const uint64_t ordinal = ex->next_invocation++;
    observe(ex, MG_OBSERVATION_DISPATCH_STARTED, inv->kernel, ordinal, MG_OK);
    // src/executor.rs:1202-1210: an already-expired deadline is a timeout.
    if (inv->deadline_millis == 0) {
        ex->failed++;
        observe(ex, MG_OBSERVATION_TIMEOUT, inv->kernel, ordinal, MG_KERNEL_TIMEOUT);
        return fail(MG_KERNEL_TIMEOUT, "kernel '%s' deadline expired before dispatch", inv->kernel);
    }
    mg_status s = device_check(ex->handle);
    if (s != MG_OK) {
        ex->failed++;
        observe(ex, MG_OBSERVATION_DISPATCH_FAILED, inv->kernel, ordinal, s);
        return s;
    }
    const std::string out_id = inv->output;
    // Offer the output id's previous buffer unless the invocation also reads it.
    mg_buffer* offered = nullptr;
    bool reads_output = false;
    for (int i = 0; i < inv->input_count; i++)
        if (inv->inputs && inv->inputs[i] && out_id == inv->inputs[i]) reads_output = true;
    auto prev = ex->storage.find(out_id);
    // Kernels that fail on data after writing (an invalid embedding id, a non-finite softmax
    // row) get a fresh buffer, so that a failure leaves the previous value intact.
    const bool data_checked = !strcmp(inv->kernel, "embedding") || !strcmp(inv->kernel, "softmax");
    if (prev != ex->storage.end() && !reads_output && !data_checked && prev->second->owned) offered = H(prev->second);
    mg_buffer* result = offered;
    const int role = ex->comm ? tp_role(ex, inv) : 0;
    // During a step capture (one rank), projections of one input are grouped into one launch.
    const bool taken = ex->capturing && !ex->comm && capture_defer(ex, inv, offered, &result, &s);
    if (!taken) {
        s = flush_deferred(ex);
        if (s == MG_OK) s = dispatch(ex, inv, &result);
        if (s == MG_OK && role == 2) s = comm_all_reduce_buffer(ex->comm, buf(result));
    }
    if (s != MG_OK) {
        // The previous value stays; a fresh buffer made for this call is dropped.
        if (result && result != offered) buffer_free(buf(result));
        ex->failed++;
        // src/executor.rs:2095-2130: an output the device cannot hold is a memory-feasibility
        // failure.
        if (s == MG_OUT_OF_DEVICE_MEMORY) observe(ex, MG_OBSERVATION_MEMORY_FEASIBILITY_FAILED, inv->kernel, ordinal, s);
        observe(ex, MG_OBSERVATION_DISPATCH_FAILED, inv->kernel, ordinal, s);
        return s;
    }
    store_replace(ex, out_id, buf(result));
    if (ex->capturing) {
        // The step records what the invocation read and wrote (src/executor.rs
        // record_captured_resources); an embedding's ids are checked on the host when a replay
        // writes them.
        for (int i = 0; i < inv->input_count; i++) {
            if (!inv->inputs || !inv->inputs[i]) continue;
            auto it = ex->storage.find(inv->inputs[i]);
            if (it != ex->storage.end()) capture_record(ex, inv->inputs[i], it->second);
        }
        capture_record(ex, out_id, buf(result));
        if (!strcmp(inv->kernel, "embedding") && inv->input_count >= 2 && inv->inputs[0] && inv->inputs[1]) {
            auto t = ex->storage.find(inv->inputs[0]);
            if (t != ex->storage.end() && t->second->rank >= 1) ex->capture_embedding_ids[inv->inputs[1]] = t->second->shape[0];
        }
    }
    if (role == 1) ex->sharded.insert(out_id);
    else ex->sharded.erase(out_id);
    ex->completed++;
    observe(ex, MG_OBSERVATION_DISPATCH_COMPLETED, inv->kernel, ordinal, MG_OK);
    return MG_OK;
}

mg_status mg_executor_synchronize(mg_executor* ex) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    return mg_device_synchronize(ex->handle);
}

mg_status mg_executor_begin_step_capture(mg_executor* ex) {
    return mg_executor_begin_step_capture_advancing(ex, nullptr, 0);
}

mg_status mg_executor_begin_step_capture_advancing(mg_executor* ex, const char* const* attributes, int count) {
    if (!ex || (count > 0 && !attributes)) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    if (ex->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "a step capture is already in progress");
    MG_TRY(device_check(ex->handle));
    Device* d = ex->device;
    if (d->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "another executor of this device is capturing a step");
    MG_CUDA(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed), "beginning a step capture");
    ex->capturing = true;
    d->capturing = true;
    graph_take(d);  // starts an empty record of the blocks the step addresses
    ex->advancing.clear();
    for (int i = 0; i < count; i++)
        if (attributes[i]) ex->advancing.insert(attributes[i]);
    ex->capture_max_offset = UINT64_MAX;
    ex->capture_has_embedding = false;
    ex->capture_resources.clear();
    ex->capture_embedding_ids.clear();
    ex->launches_at_capture = d->launches.load();
    return MG_OK;
}

namespace {

// Ends the capture in progress and instantiates its graph (src/executor.rs end_step_capture).
mg_status end_capture(mg_executor* ex, CapturedStep** out) {
    *out = nullptr;
    if (!ex->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "no step capture is in progress");
    Device* d = ex->device;
    const mg_status fs = flush_deferred(ex);  // the last deferred group
    cudaGraph_t gph = nullptr;
    cudaError_t e = cudaStreamEndCapture(d->stream, &gph);
    ex->capturing = d->capturing = false;
    // The blocks the graph addresses are held before the frees deferred during the capture run,
    // so a block the capture both used and released stays allocated for the graph.
    CapturedStep* st = new (std::nothrow) CapturedStep();
    if (!st) {
        if (gph) cudaGraphDestroy(gph);
        graph_take(d);
        flush_deferred_frees(d);
        return fail(MG_EXECUTION_FAILED, "host allocation failed");
    }
    st->blocks = graph_take(d);
    graph_hold(d, st->blocks);
    flush_deferred_frees(d);
    const uint64_t kernels = d->launches.load() - ex->launches_at_capture;
    d->launches.fetch_sub(kernels);  // captured launches did not run; replays count them
    if (e != cudaSuccess || fs != MG_OK) {
        st->graph = gph;
        step_destroy(ex, st);
        return fs != MG_OK ? fs : from_cuda(e, "ending the step capture");
    }
    st->graph = gph;
    e = cudaGraphInstantiate(&st->exec, gph, 0);
    if (e != cudaSuccess) {
        st->exec = nullptr;
        step_destroy(ex, st);
        return from_cuda(e, "instantiating the step graph");
    }
    st->kernels = kernels;
    st->advancing = !ex->advancing.empty();
    st->max_offset = ex->capture_max_offset;
    st->has_embedding = ex->capture_has_embedding;
    st->resources.swap(ex->capture_resources);
    st->embedding_ids.swap(ex->capture_embedding_ids);
    st->storage_gen = ex->storage_gen;
    st->prep_gen = d->prep_gen.load();
    ex->advancing.clear();
    *out = st;
    return MG_OK;
}

// Whether every resource the step recorded still has its captured storage (src/executor.rs
// replay_step: "resource '...' no longer has its captured storage"), including the operand
// forms of weights its matmuls read.
mg_status step_check_storage(mg_executor* ex, CapturedStep* st) {
    const uint64_t pg = ex->device->prep_gen.load();
    if (st->storage_gen == ex->storage_gen && st->prep_gen == pg) return MG_OK;
    for (const auto& kv : st->resources) {
        auto it = ex->storage.find(kv.first);
        const CapturedStep::Resource& r = kv.second;
        const Buffer* b = it == ex->storage.end() ? nullptr : it->second;
        if (!b || b != r.b || b->ptr != r.ptr || b->count != r.count)
            return fail(MG_CAPTURE_UNSUPPORTED, "resource '%s' no longer has its captured storage", kv.first.c_str());
        if ((r.prep && b->prep != r.prep) || (r.compact && b->compact != r.compact))
            return fail(MG_CAPTURE_UNSUPPORTED,
                        "resource '%s' changed after the capture: the operand form the step reads is gone; capture the step again",
                        kv.first.c_str());
    }
    st->storage_gen = ex->storage_gen;
    st->prep_gen = pg;
    return MG_OK;
}

CapturedStep* find_step(mg_executor* ex, uint64_t id) {
    auto it = ex->steps.find(id);
    return it == ex->steps.end() ? nullptr : it->second;
}

// Reads (and resets) the sticky embedding-id flag after replays; waits for the device.
mg_status check_embedding_flag(Device* d) {
    MG_CUDA(cudaMemcpyAsync(d->host_flags, d->flags, sizeof(int), cudaMemcpyDeviceToHost, d->stream), "reading the id flag");
    MG_CUDA(cudaMemsetAsync(d->flags, 0, sizeof(int), d->stream), "resetting the id flag");
    MG_CUDA(cudaStreamSynchronize(d->stream), "waiting for the replayed step");
    if (d->host_flags[0])
        return fail(MG_SHAPE_UNSUPPORTED, "embedding lookup id is not a valid in-range non-negative integer");
    return MG_OK;
}

// Replays `st` `count` times at `offset` (count < 0: one launch and no check; 0: the check
// only).
mg_status replay_step_n(mg_executor* ex, CapturedStep* st, int count, uint64_t offset) {
    Device* d = ex->device;
    if (offset > st->max_offset)
        return fail(MG_CAPTURE_UNSUPPORTED, "offset %llu leaves the captured bounds (at most %llu)",
                    (unsigned long long)offset, (unsigned long long)st->max_offset);
    const int launches = count < 0 ? 1 : count;
    if (launches > 0) MG_TRY(step_check_storage(ex, st));
    if (st->advancing && launches > 0) MG_TRY(k::set_step_offset(d, d->step_offset, offset));
    for (int i = 0; i < launches; i++) {
        MG_CUDA(cudaGraphLaunch(st->exec, d->stream), "replaying the captured step");
        d->launches.fetch_add(st->kernels);
    }
    if (count < 0) return MG_OK;
    // The id flag is sticky across the replays: one read covers them all, then resets.
    if (st->has_embedding) return check_embedding_flag(d);
    return MG_OK;
}

bool pinned_host(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// The address the GPU reaches page-locked host memory at (null: not mapped).
void* mapped_host(void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// A replay's host copy done by the SMs over the mapped address instead of a copy-engine node:
// a copy engine spends several microseconds starting even a small transfer (256 KB device to
// host: ~15 us with its synchronisation), while the SMs' loads and stores to host memory go out
// at once.  16 bytes per thread where both ends are 16-byte aligned, bytes otherwise.  With
// `flag`, the first thread also moves the device's sticky embedding-id word to the host word
// and clears it (the replay's flag read and reset).  One system-scope fence per block, after the
// block's barrier, orders all of the block's stores (fences are cumulative); a fence in every
// thread made a 256 KB copy ~3 us slower after the step's last kernel (14.4 against 11.5 us).
__global__ void __launch_bounds__(256) io_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                      uint64_t bytes, int* flag, int* flag_host) {
    // An output copy hangs off the step's last kernels by programmatic edges: it is scheduled
    // while they finish and waits here for their completion and memory (at once otherwise).  An
    // input copy lets the step's first kernels be scheduled while it runs; they wait for it in
    // their own pdl_enter().
    pdl_enter();
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (uint64_t)gridDim.x * blockDim.x;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    const uint64_t n16 = vec ? bytes / 16 : 0;
    for (uint64_t i = tid; i < n16; i += nth) reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    for (uint64_t i = n16 * 16 + tid; i < bytes; i += nth) dst[i] = src[i];
    if (flag && tid == 0) {
        *flag_host = *flag;
        *flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// The nodes of `graph` without dependencies and those without dependents.
bool graph_ends(cudaGraph_t graph, std::vector<cudaGraphNode_t>& roots, std::vector<cudaGraphNode_t>& leaves) {
    size_t n = 0;
    if (cudaGraphGetNodes(graph, nullptr, &n) != cudaSuccess) return false;
    std::vector<cudaGraphNode_t> nodes(n);
    if (n && cudaGraphGetNodes(graph, nodes.data(), &n) != cudaSuccess) return false;
    for (cudaGraphNode_t node : nodes) {
        size_t in = 0, out = 0;
        if (cudaGraphNodeGetDependencies(node, nullptr, &in) != cudaSuccess ||
            cudaGraphNodeGetDependentNodes(node, nullptr, &out) != cudaSuccess)
            return false;
        if (!in) roots.push_back(node);
        if (!out) leaves.push_back(node);
    }
    return true;
}

// Whether every kernel node of `graph` is one of the library's own launches: the step counted
// `kernels` of them while it was captured, and each starts with pdl_enter(), so it waits for an
// upstream grid before it reads memory and may take a programmatic edge.  (A step captured under
// a tensor-parallel plan also holds the communication library's kernels.)
bool only_library_kernels(cudaGraph_t graph, uint64_t kernels) {
    size_t n = 0;
    if (cudaGraphGetNodes(graph, nullptr, &n) != cudaSuccess) return false;
    std::vector<cudaGraphNode_t> nodes(n);
    if (n && cudaGraphGetNodes(graph, nodes.data(), &n) != cudaSuccess) return false;
    uint64_t count = 0;
    for (cudaGraphNode_t node : nodes) {
        cudaGraphNodeType type;
        if (cudaGraphNodeGetType(node, &type) != cudaSuccess) return false;
        count += type == cudaGraphNodeTypeKernel;
    }
    return count == kernels;
}

// Edges from each of `from` to `to`.  With `to_waits` (`to` is a kernel node that starts with
// pdl_enter()) an edge from a kernel node is programmatic, so `to` is scheduled while that kernel
// finishes and waits for it in the kernel; every other edge is a plain one.
bool add_edges(cudaGraph_t graph, const std::vector<cudaGraphNode_t>& from, cudaGraphNode_t to, bool to_waits) {
    for (cudaGraphNode_t f : from) {
        cudaGraphEdgeData e = {};
        cudaGraphNodeType type;
        if (cudaGraphNodeGetType(f, &type) != cudaSuccess) return false;
        if (to_waits && type == cudaGraphNodeTypeKernel) {
            e.from_port = cudaGraphKernelNodePortProgrammatic;
            e.type = cudaGraphDependencyTypeProgrammatic;
        }
        if (cudaGraphAddDependencies_v2(graph, &f, &to, &e, 1) != cudaSuccess) return false;
    }
    return true;
}

// Adds an io_copy_kernel node copying `bytes` from src to dst after `deps`.
bool add_io_copy(cudaGraph_t graph, const cudaGraphNode_t* deps, size_t ndeps, const void* src, void* dst,
                 uint64_t bytes, int* flag, int* flag_host, cudaGraphNode_t* node) {
    const uint64_t chunks = (bytes + 15) / 16;
    unsigned grid = (unsigned)std::min<uint64_t>(148, std::max<uint64_t>(1, (chunks + 255) / 256));
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint8_t* d = static_cast<uint8_t*>(dst);
    void* args[] = {(void*)&s, (void*)&d, (void*)&bytes, (void*)&flag, (void*)&flag_host};
    cudaKernelNodeParams kp = {};
    kp.func = (void*)io_copy_kernel;
    kp.gridDim = dim3(grid);
    kp.blockDim = dim3(256);
    kp.sharedMemBytes = 0;
    kp.kernelParams = args;
    return cudaGraphAddKernelNode(node, graph, deps, ndeps, &kp) == cudaSuccess;
}

// The one-launch graph of a replay with this host I/O (built on first use, kept with the step):
// null when some host buffer is not pinned (graph copies need page-locked memory) or the graph
// cannot be built, in which case the replay issues its copies separately.
CapturedStep::IoGraph* io_graph_for(mg_executor* ex, CapturedStep* st, const mg_step_io* io, int count,
                                    const std::vector<Buffer*>& bufs) {
    for (CapturedStep::IoGraph* g : st->io_graphs) {
        if ((int)g->io.size() != count) continue;
        bool same = true;
        for (int i = 0; i < count && same; i++)
            same = g->io[i].host == io[i].host && g->io[i].bytes == io[i].bytes && g->io[i].to_device == io[i].to_device &&
                   g->names[i] == io[i].id && g->device[i] == bufs[(size_t)i]->ptr;
        if (same) return g;
    }
    for (int i = 0; i < count; i++)
        if (io[i].bytes && !pinned_host(io[i].host)) return nullptr;
    Device* d = ex->device;
    CapturedStep::IoGraph* g = new (std::nothrow) CapturedStep::IoGraph();
    if (!g) return nullptr;
    // The step's own nodes, cloned (not nested as a child graph, whose nodes no edge can reach):
    // the input copies come before its first nodes, the output copies after its last kernels.
    bool ok = cudaGraphClone(&g->graph, st->graph) == cudaSuccess;
    std::vector<cudaGraphNode_t> roots, leaves;
    if (ok) ok = graph_ends(g->graph, roots, leaves);
    const bool roots_wait = ok && only_library_kernels(g->graph, st->kernels);
    std::vector<cudaGraphNode_t> before;
    for (int i = 0; ok && i < count; i++) {
        g->names.push_back(io[i].id);
        g->io.push_back(io[i]);
        g->device.push_back(bufs[(size_t)i]->ptr);
        if (!io[i].to_device || !io[i].bytes) continue;
        cudaGraphNode_t n;
        void* mh = mapped_host(io[i].host);
        if (mh)
            ok = add_io_copy(g->graph, nullptr, 0, mh, bufs[(size_t)i]->ptr, io[i].bytes, nullptr, nullptr, &n);
        else
            ok = cudaGraphAddMemcpyNode1D(&n, g->graph, nullptr, 0, bufs[(size_t)i]->ptr, io[i].host, io[i].bytes,
                                          cudaMemcpyHostToDevice) == cudaSuccess;
        if (ok) before.push_back(n);
    }
    if (ok && st->advancing) {
        ok = cudaMallocHost(&g->offset_word, sizeof(uint64_t)) == cudaSuccess;
        cudaGraphNode_t n;
        if (ok)
            ok = cudaGraphAddMemcpyNode1D(&n, g->graph, nullptr, 0, d->step_offset, g->offset_word, sizeof(uint64_t),
                                          cudaMemcpyHostToDevice) == cudaSuccess;
        if (ok) before.push_back(n);
    }
    for (size_t r = 0; ok && r < roots.size(); r++) {
        cudaGraphNodeType type;
        ok = cudaGraphNodeGetType(roots[r], &type) == cudaSuccess &&
             add_edges(g->graph, before, roots[r], roots_wait && type == cudaGraphNodeTypeKernel);
    }
    // what the output copies follow: the step's last nodes (the input copies for an empty step)
    const std::vector<cudaGraphNode_t>& last = leaves.empty() ? before : leaves;
    // The embedding-id word rides along with the first output copy done by the SMs.
    int* flag_host = st->has_embedding ? static_cast<int*>(mapped_host(d->host_flags)) : nullptr;
    bool flag_done = false;
    for (int i = 0; ok && i < count; i++) {
        if (io[i].to_device || !io[i].bytes) continue;
        cudaGraphNode_t n;
        void* mh = mapped_host(io[i].host);
        if (mh) {
            const bool with_flag = flag_host && !flag_done;
            ok = add_io_copy(g->graph, nullptr, 0, bufs[(size_t)i]->ptr, mh, io[i].bytes, with_flag ? d->flags : nullptr,
                             with_flag ? flag_host : nullptr, &n) &&
                 add_edges(g->graph, last, n, true);
            flag_done = flag_done || with_flag;
        } else {
            ok = cudaGraphAddMemcpyNode1D(&n, g->graph, nullptr, 0, io[i].host, bufs[(size_t)i]->ptr, io[i].bytes,
                                          cudaMemcpyDeviceToHost) == cudaSuccess &&
                 add_edges(g->graph, last, n, false);
        }
    }
    if (ok && flag_host && !flag_done) {
        cudaGraphNode_t n;
        ok = add_io_copy(g->graph, nullptr, 0, nullptr, nullptr, 0, d->flags, flag_host, &n) && add_edges(g->graph, last, n, true);
        flag_done = ok;
    }
    if (ok && st->has_embedding && !flag_done) {
        // the sticky id flag read back, then reset for the next replay
        cudaGraphNode_t rd, rs;
        ok = cudaGraphAddMemcpyNode1D(&rd, g->graph, nullptr, 0, d->host_flags, d->flags, sizeof(int),
                                      cudaMemcpyDeviceToHost) == cudaSuccess &&
             add_edges(g->graph, last, rd, false);
        cudaMemsetParams mp = {};
        mp.dst = d->flags;
        mp.value = 0;
        mp.elementSize = sizeof(int);
        mp.width = 1;
        mp.height = 1;
        if (ok) ok = cudaGraphAddMemsetNode(&rs, g->graph, &rd, 1, &mp) == cudaSuccess;
    }
    if (ok) ok = cudaGraphInstantiate(&g->exec, g->graph, 0) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        io_graph_destroy(g);
        st->io_graph_failed = true;
        return nullptr;
    }
    if (st->io_graphs.size() >= 4) {  // a few host-buffer sets per step; the oldest goes
        io_graph_destroy(st->io_graphs.front());
        st->io_graphs.erase(st->io_graphs.begin());
    }
    st->io_graphs.push_back(g);
    return g;
}

// One replay with host I/O (see mg_executor_replay_step_io).
mg_status replay_io(mg_executor* ex, CapturedStep* st, uint64_t offset, const mg_step_io* io, int count) {
    Device* d = ex->device;
    if (offset > st->max_offset)
        return fail(MG_CAPTURE_UNSUPPORTED, "offset %llu leaves the captured bounds (at most %llu)",
                    (unsigned long long)offset, (unsigned long long)st->max_offset);
    MG_TRY(step_check_storage(ex, st));
    std::vector<Buffer*> bufs((size_t)count);
    for (int i = 0; i < count; i++) {
        if (!io[i].id || (!io[i].host && io[i].bytes)) return fail(MG_INVALID_ARGUMENT, "null argument");
        auto it = ex->storage.find(io[i].id);
        if (it == ex->storage.end()) return fail(MG_EXECUTION_FAILED, "no materialized data for resource %s", io[i].id);
        Buffer* b = it->second;
        if (b->dtype == MG_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "resource %s is a packed weight", io[i].id);
        if (io[i].bytes != b->count * dtype_size(b->dtype))
            return fail(MG_SHAPE_UNSUPPORTED, "%llu bytes do not match resource %s of shape %s",
                        (unsigned long long)io[i].bytes, io[i].id, shape_str(b).c_str());
        if (io[i].to_device) {
            auto r = st->resources.find(io[i].id);
            // src/executor.rs replay_step: an input the step never read is refused.
            if (r == st->resources.end())
                return fail(MG_CAPTURE_UNSUPPORTED, "input '%s' was not read by the captured step", io[i].id);
            // The step reads this weight through an operand form derived from its values: new
            // values would not reach it.
            if (r->second.prep || r->second.compact)
                return fail(MG_CAPTURE_UNSUPPORTED,
                            "input '%s' is a weight the captured step reads through its operand form; write it with "
                            "write_weight_tensor and capture the step again",
                            io[i].id);
            auto e = st->embedding_ids.find(io[i].id);
            if (e != st->embedding_ids.end() && b->dtype == MG_F32) {  // src/executor.rs replay_step
                const float* v = (const float*)io[i].host;
                for (uint64_t j = 0; j < b->count; j++)
                    if (!(v[j] >= 0.0f && v[j] == std::floor(v[j]) && (uint64_t)v[j] < e->second))
                        return fail(MG_SHAPE_UNSUPPORTED, "embedding lookup id is not a valid in-range non-negative integer");
            }
        }
        bufs[(size_t)i] = b;
    }
    if (!st->io_graph_failed) {
        CapturedStep::IoGraph* g = io_graph_for(ex, st, io, count, bufs);
        if (g) {
            if (g->offset_word) *g->offset_word = offset;  // read by the graph's first copy
            MG_CUDA(cudaGraphLaunch(g->exec, d->stream), "replaying the captured step");
            d->launches.fetch_add(st->kernels);
            for (int i = 0; i < count; i++) (io[i].to_device ? d->uploads : d->downloads).fetch_add(io[i].bytes ? 1 : 0);
            MG_CUDA(cudaStreamSynchronize(d->stream), "waiting for the replayed step");
            if (st->has_embedding && d->host_flags[0])
                return fail(MG_SHAPE_UNSUPPORTED, "embedding lookup id is not a valid in-range non-negative integer");
            return MG_OK;
        }
    }
    for (int i = 0; i < count; i++) {
        if (!io[i].to_device || !io[i].bytes) continue;
        MG_CUDA(cudaMemcpyAsync(bufs[(size_t)i]->ptr, io[i].host, io[i].bytes, cudaMemcpyHostToDevice, d->stream),
                "writing a step input");
        d->uploads.fetch_add(1);
    }
    if (st->advancing) MG_TRY(k::set_step_offset(d, d->step_offset, offset));
    MG_CUDA(cudaGraphLaunch(st->exec, d->stream), "replaying the captured step");
    d->launches.fetch_add(st->kernels);
    for (int i = 0; i < count; i++) {
        if (io[i].to_device || !io[i].bytes) continue;
        MG_CUDA(cudaMemcpyAsync(io[i].host, bufs[(size_t)i]->ptr, io[i].bytes, cudaMemcpyDeviceToHost, d->stream),
                "reading a step output");
        d->downloads.fetch_add(1);
    }
    if (st->has_embedding) return check_embedding_flag(d);
    MG_CUDA(cudaStreamSynchronize(d->stream), "waiting for the replayed step");
    return MG_OK;
}

}  // namespace

mg_status mg_executor_end_step_capture(mg_executor* ex) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = nullptr;
    MG_TRY(end_capture(ex, &st));
    // The single-step calls' step: replaces the previous one made by this call.
    if (ex->current) {
        step_destroy(ex, find_step(ex, ex->current));
        ex->steps.erase(ex->current);
    }
    ex->current = ex->next_step++;
    ex->steps[ex->current] = st;
    return MG_OK;
}

mg_status mg_executor_end_step_capture_id(mg_executor* ex, uint64_t* id) {
    if (!ex || !id) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = nullptr;
    MG_TRY(end_capture(ex, &st));
    // src/executor.rs end_step_capture: the captured graph runs once as it ends, so the
    // captured step's results are available.
    const mg_status s = replay_step_n(ex, st, 1, 0);
    if (s != MG_OK) {
        step_destroy(ex, st);
        return s;
    }
    *id = ex->next_step++;
    ex->steps[*id] = st;
    return MG_OK;
}

mg_status mg_executor_replay_capture(mg_executor* ex, uint64_t id, uint64_t offset, const mg_step_io* io, int count) {
    if (!ex || (count > 0 && !io) || count < 0) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = find_step(ex, id);
    if (!st) return fail(MG_CAPTURE_UNSUPPORTED, "no step capture %llu", (unsigned long long)id);
    MG_TRY(device_check(ex->handle));
    return replay_io(ex, st, offset, io, count);
}

mg_status mg_executor_release_step_capture(mg_executor* ex, uint64_t id) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    auto it = ex->steps.find(id);
    if (it == ex->steps.end()) return MG_OK;
    step_destroy(ex, it->second);
    ex->steps.erase(it);
    if (ex->current == id) ex->current = 0;
    return MG_OK;
}

mg_status mg_executor_step_capture_count(mg_executor* ex, int* count) {
    if (!ex || !count) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    *count = (int)ex->steps.size();
    return MG_OK;
}

mg_status mg_executor_abort_step_capture(mg_executor* ex) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    if (!ex->capturing) return MG_OK;
    cudaGraph_t gph = nullptr;
    ex->deferred.clear();
    ex->deferred_rope = false;
    ex->embed_pending = false;
    ex->advancing.clear();
    ex->capture_resources.clear();
    ex->capture_embedding_ids.clear();
    cudaStreamEndCapture(ex->device->stream, &gph);
    cudaGetLastError();
    if (gph) cudaGraphDestroy(gph);
    ex->capturing = ex->device->capturing = false;
    graph_take(ex->device);
    flush_deferred_frees(ex->device);
    ex->device->launches.fetch_sub(ex->device->launches.load() - ex->launches_at_capture);
    return MG_OK;
}

namespace {
// The single-step calls: the step mg_executor_end_step_capture made last.
mg_status replay_at(mg_executor* ex, int count, uint64_t offset) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = find_step(ex, ex->current);
    if (!st) return fail(MG_CAPTURE_UNSUPPORTED, "no captured step to replay");
    MG_TRY(device_check(ex->handle));
    return replay_step_n(ex, st, count, offset);
}

}  // namespace

mg_status mg_executor_replay_steps(mg_executor* ex, int count) { return replay_at(ex, count, 0); }

// src/executor.rs replay_step(id, offset, inputs) with the step's outputs read in the same call:
// the inputs' host bytes are copied into their captured buffers, the step replays at `offset`,
// the outputs are copied out, and one synchronisation covers them and the embedding-id check.
mg_status mg_executor_replay_step_io(mg_executor* ex, uint64_t offset, const mg_step_io* io, int count) {
    if (!ex || (count > 0 && !io) || count < 0) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = find_step(ex, ex->current);
    if (!st) return fail(MG_CAPTURE_UNSUPPORTED, "no captured step to replay");
    MG_TRY(device_check(ex->handle));
    return replay_io(ex, st, offset, io, count);
}

mg_status mg_executor_replay_step_at(mg_executor* ex, uint64_t offset) { return replay_at(ex, 1, offset); }

mg_status mg_executor_step_max_offset(mg_executor* ex, uint64_t* out) {
    if (!ex || !out) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    CapturedStep* st = find_step(ex, ex->current);
    if (!st) return fail(MG_CAPTURE_UNSUPPORTED, "no captured step");
    *out = st->max_offset;
    return MG_OK;
}

mg_status mg_executor_replay_step(mg_executor* ex) { return mg_executor_replay_steps(ex, 1); }

mg_status mg_executor_launch_step(mg_executor* ex) { return mg_executor_replay_steps(ex, -1); }

mg_status mg_executor_check_steps(mg_executor* ex) { return mg_executor_replay_steps(ex, 0); }

mg_status mg_executor_observations(mg_executor* ex, uint64_t* started, uint64_t* completed, uint64_t* failed) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    if (started) *started = ex->started;
    if (completed) *completed = ex->completed;
    if (failed) *failed = ex->failed;
    return MG_OK;
}

mg_status mg_executor_observation_log(mg_executor* ex, mg_observation* out, uint32_t capacity, uint32_t* count) {
    if (!ex || !count || (capacity && !out)) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    const size_t held = ex->observations.size();
    const size_t first = held > MG_OBSERVATION_LOG_CAPACITY ? held - MG_OBSERVATION_LOG_CAPACITY : 0;
    const size_t n = held - first;
    *count = (uint32_t)n;
    if (!out) return MG_OK;
    if (capacity < n)
        return fail(MG_SHAPE_UNSUPPORTED, "%u entries cannot hold the %zu observations", capacity, n);
    for (size_t i = 0; i < n; i++) {
        const Observation& o = ex->observations[first + i];
        mg_observation& r = out[i];
        memset(&r, 0, sizeof r);
        r.kind = o.kind;
        snprintf(r.kernel, sizeof r.kernel, "%s", o.kernel.c_str());
        r.invocation = o.invocation;
        r.status = o.status;
    }
    return MG_OK;
}

mg_status mg_executor_attach_comm(mg_executor* ex, mg_comm* comm) {
    if (!ex) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    ex->comm = comm;
    return MG_OK;
}

mg_status mg_executor_apply_tensor_parallel(mg_executor* ex, int count, const char* const* ids, const int* kinds) {
    if (!ex || (count > 0 && (!ids || !kinds))) return fail(MG_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> g(ex->lock);
    if (!ex->comm) return fail(MG_EXECUTION_FAILED, "a tensor-parallel plan needs a communicator (mg_executor_attach_comm)");
    for (int i = 0; i < count; i++)
        if (kinds[i] != 0 && kinds[i] != 1) return fail(MG_ATTRIBUTE_UNSUPPORTED, "weight shard kind %d is not implemented", kinds[i]);
    ex->plan.clear();
    for (int i = 0; i < count; i++) ex->plan[ids[i]] = kinds[i];
    return MG_OK;
}

}  // extern "C"
