// Host runtime of the B200 training hot path: NodeBackProp, AdamParameter,
// GraphOperations and Linear with the reference's API (Includes/engine.h),
// launching only through the C ABI of include/mle_kernels.h.
//
// Each builder cites the reference lambda whose semantics it keeps.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <random>
#include <unordered_map>
#include <unordered_set>

#include "engine.h"
#include "engine_internal.h"

// ============================================================================
// runtime: stream, errors, arenas, coalesced zeroing, parameter registry
// ============================================================================
namespace mle {

static cudaStream_t g_stream = 0;
cudaStream_t stream() { return g_stream; }
void set_stream(cudaStream_t s) { g_stream = s; }
void* st() { return (void*)g_stream; }

static bool g_ps_enabled = true;
static cudaStream_t g_ps = nullptr;
static cudaEvent_t g_ps_fork = nullptr, g_ps_join = nullptr;
static bool g_ps_pending = false;

void init_param_stream() {
    if (g_ps) return;
    check_cuda(cudaStreamCreateWithFlags(&g_ps, cudaStreamNonBlocking), "param stream");
    check_cuda(cudaEventCreateWithFlags(&g_ps_fork, cudaEventDisableTiming), "param stream");
    check_cuda(cudaEventCreateWithFlags(&g_ps_join, cudaEventDisableTiming), "param stream");
}

cudaStream_t fork_param_stream() {
    if (!g_ps_enabled) return g_stream;
    init_param_stream();
    check_cuda(cudaEventRecord(g_ps_fork, g_stream), "param stream fork");
    check_cuda(cudaStreamWaitEvent(g_ps, g_ps_fork, 0), "param stream fork");
    g_ps_pending = true;
    return g_ps;
}

void join_param_stream() {
    if (!g_ps_pending) return;
    check_cuda(cudaEventRecord(g_ps_join, g_ps), "param stream join");
    check_cuda(cudaStreamWaitEvent(g_stream, g_ps_join, 0), "param stream join");
    g_ps_pending = false;
}

bool param_stream_pending() { return g_ps_pending; }
cudaStream_t param_stream() { return g_ps; }
void set_param_stream_enabled(bool on) {
    join_param_stream();
    g_ps_enabled = on;
}
bool param_stream_enabled() { return g_ps_enabled; }

void check(int status, const str& what) {
    if (status != MLE_OK) {
        std::cerr << "Runtime error in " << what << ": " << mle_status_string(status)
                  << " (cuda error " << mle_last_cuda_error() << ")" << std::endl;
        std::exit(1);
    }
}

void check_cuda(cudaError_t e, const str& what) {
    if (e != cudaSuccess) {
        std::cerr << "CUDA error in " << what << ": " << cudaGetErrorString(e) << std::endl;
        std::exit(1);
    }
}

struct ArenaChunk {
    char* base;
    int64_t size, used;
};

static std::vector<ArenaChunk> g_arenas[ARENA_COUNT];
static constexpr int64_t kChunk = 256ll << 20;

void* arena_alloc_bytes(Arena a, int64_t bytes, const str& name) {
    if (bytes <= 0) bytes = 4;
    const int64_t need = (bytes + 255) & ~int64_t(255);
    auto& chunks = g_arenas[a];
    if (chunks.empty() || chunks.back().size - chunks.back().used < need) {
        const int64_t sz = std::max(kChunk, need);
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, (size_t)sz);
        if (e != cudaSuccess) {
            size_t fr = 0, tot = 0;
            cudaMemGetInfo(&fr, &tot);
            std::cerr << "Failed to allocate " << name << " of size " << bytes << ": " << cudaGetErrorString(e)
                      << std::endl;
            std::cout << "GPU memory free: " << (fr >> 20) << " MB of " << (tot >> 20) << " MB\n";
            std::exit(1);
        }
        // graph-build time: new chunks start zeroed (grads rely on it)
        check_cuda(cudaMemset(p, 0, (size_t)sz), "arena zero-fill");
        chunks.push_back({(char*)p, sz, 0});
    }
    ArenaChunk& c = chunks.back();
    char* out = c.base + c.used;
    c.used += need;
    return out;
}

float* arena_alloc(Arena a, int64_t n_floats, const str& name) {
    return (float*)arena_alloc_bytes(a, n_floats * (int64_t)sizeof(float), name);
}

double arena_gib(Arena a) {
    double s = 0;
    for (auto& c : g_arenas[a]) s += (double)c.used;
    return s / (double)(1ull << 30);
}

void release_all_arenas() {
    for (auto& v : g_arenas) {
        for (auto& c : v) cudaFree(c.base);
        v.clear();
    }
}

// ----------------------------------------------------------- zero batching
static int g_zero_depth = 0;
static std::vector<std::pair<float*, int64_t>> g_zero_ranges;

// Base of the arena chunk holding p (nullptr if none): ranges merge only
// within one chunk, since two chunks that happen to be adjacent in the
// address space are still separate allocations a memset may not span.
static const char* chunk_base(const void* p) {
    const char* c = static_cast<const char*>(p);
    for (auto& v : g_arenas)
        for (auto& ch : v)
            if (c >= ch.base && c < ch.base + ch.size) return ch.base;
    return nullptr;
}

const void* arena_chunk_of(const void* p) { return chunk_base(p); }

static void flush_zero_ranges() {
    auto& r = g_zero_ranges;
    if (r.empty()) return;
    std::sort(r.begin(), r.end());
    float* cur = r[0].first;
    int64_t len = r[0].second;
    auto emit = [](float* p, int64_t n) {
        check_cuda(cudaMemsetAsync(p, 0, (size_t)n * sizeof(float), g_stream), "zero_grad");
    };
    for (size_t i = 1; i < r.size(); ++i) {
        float* p = r[i].first;
        const int64_t n = r[i].second;
        // merge if the next range starts inside or at most one alignment pad
        // (<= 256 bytes) after the current one: the pad bytes belong to no
        // buffer, so clearing them is harmless
        if (p <= cur + len + 64 && chunk_base(p) == chunk_base(cur)) {
            const int64_t end = std::max<int64_t>((p + n) - cur, len);
            len = end;
        } else {
            emit(cur, len);
            cur = p;
            len = n;
        }
    }
    emit(cur, len);
    r.clear();
}

// Gradients whose first writer in the backward assigns them, for the graph
// whose fusions were planned last.  zero_range consults the set only inside
// GraphOperations::zero_grad, which plans its own graph first, so a graph
// never skips a buffer on the strength of another graph's plan (two graphs
// may share nodes, and one may assign a gradient the other accumulates).
static std::unordered_set<const float*> g_preassigned;
static bool g_first_write = true;
static int g_skip_depth = 0;

void set_preassigned_grads(const std::vector<const float*>& grads) {
    g_preassigned.clear();
    if (g_first_write) g_preassigned.insert(grads.begin(), grads.end());
}

bool grad_preassigned(const float* grad) { return g_preassigned.count(grad) != 0; }

void set_first_write_assign(bool on) {
    g_first_write = on;
    if (!on) g_preassigned.clear();
}

bool first_write_assign() { return g_first_write; }

void zero_range(float* p, int64_t n) {
    if (!p || n <= 0) return;
    if (g_skip_depth > 0 && g_preassigned.count(p)) return;  // its first writer in the backward assigns it
    if (g_zero_depth > 0) g_zero_ranges.push_back({p, n});
    else check_cuda(cudaMemsetAsync(p, 0, (size_t)n * sizeof(float), g_stream), "Zerograd");
}

ZeroBatch::ZeroBatch() { ++g_zero_depth; }
ZeroBatch::~ZeroBatch() {
    if (--g_zero_depth == 0) flush_zero_ranges();
}

// --------------------------------------------------------- parameter state
std::vector<AdamParameter*>& all_parameters() {
    static std::vector<AdamParameter*> v;
    return v;
}

static uint64_t g_seed = 0;
static bool g_seeded = false;
static uint64_t g_param_counter = 0;
void set_seed(uint64_t seed) {
    g_seed = seed;
    g_seeded = true;
    g_param_counter = 0;
}

double* clip_workspace() {
    static double* ws = nullptr;
    if (!ws) ws = (double*)arena_alloc_bytes(ARENA_WS, 256, "clip workspace");
    return ws;
}

// Collection of AdamParameters touched by the per-node lambdas while a
// fused launch is being assembled.
ParamCollector* g_collector = nullptr;

bool g_keep_softmax = true;
void set_keep_softmax(bool keep) { g_keep_softmax = keep; }

}  // namespace mle

using namespace mle;

// ============================================================================
// debug helpers with the reference's behaviour
// ============================================================================
void CheckError(const str& reason) {
    cudaError_t launchErr = cudaGetLastError();
    cudaError_t syncErr = cudaDeviceSynchronize();
    if (launchErr != cudaSuccess) {
        std::cerr << "Launch error in " << reason << ": " << cudaGetErrorString(launchErr) << std::endl;
        std::exit(1);
    }
    if (syncErr != cudaSuccess) {
        std::cerr << "Runtime error in " << reason << ": " << cudaGetErrorString(syncErr) << std::endl;
        std::exit(1);
    }
}

// The reference's isNan launches a kernel that __trap()s on NaN
// (Includes/kernels.h:382-392).  Here the NaNs are counted on the device and
// the host decides: on any it prints and exits as CheckError would.
static void host_nan_check(const float* p, long long n, const str& what) {
    if (!p || n <= 0) return;
    mle::nan_check(what, p, n);
}

static void print_head(const float* p, long long n, const str& name) {
    const long long k = std::min<long long>(n, 10);
    std::vector<float> h((size_t)k);
    check_cuda(cudaStreamSynchronize(g_stream), name);
    check_cuda(cudaMemcpy(h.data(), p, (size_t)k * sizeof(float), cudaMemcpyDeviceToHost), name);
    std::cout << "Printing dimensions for pointer: " << name << "\n";
    for (auto v : h) std::cout << v << "\t";
    std::cout << "\n _______________________________ \n";
}

float ReadValueAt(const graph& X, const int& idx, const bool grad) {
    float out;
    check_cuda(cudaStreamSynchronize(g_stream), "ReadValueAt");
    check_cuda(cudaMemcpy(&out, (grad ? X->grad : X->output) + idx, sizeof(float), cudaMemcpyDeviceToHost),
               "ReadValueAt");
    return out;
}

void WriteValueAt(const graph& X, const float value, const int& idx, const bool grad) {
    check_cuda(cudaStreamSynchronize(g_stream), "WriteValueAt");
    check_cuda(cudaMemcpy((grad ? X->grad : X->output) + idx, &value, sizeof(float), cudaMemcpyHostToDevice),
               "WriteValueAt");
}

// ============================================================================
// NodeBackProp (Engine/engine.cu:45-124)
// ============================================================================
NodeBackProp::NodeBackProp(str name, int batch, int d1, int d2, int d3, int allocation) : op_name(std::move(name)) {
    dim[0] = batch;
    dim[1] = d1;
    dim[2] = d2;
    dim[3] = d3;
    total = (long long)batch * d1 * d2 * d3;
    if (allocation == 1) {  // activation node: output + grad (grad starts at 0)
        output = arena_alloc(ARENA_ACT, total, op_name);
        grad = arena_alloc(ARENA_GRAD, total, op_name + " grad");
    } else if (allocation == 2) {  // parameter: contiguous parameter arenas
        output = arena_alloc(ARENA_PARAM, total, op_name);
        grad = arena_alloc(ARENA_PARAM_GRAD, total, op_name + " grad");
    } else {
        output = nullptr;
        grad = nullptr;
    }
    node_born(this);
}

NodeBackProp::~NodeBackProp() { forget_ext(this); }

void NodeBackProp::clear() {
    // Arena memory is released with the arenas; the reference cudaFrees here.
    inputs.clear();
    op_name.clear();
}

void NodeBackProp::reshape(std::vector<int> d) {
    if (d.size() != 4) {
        std::cerr << "Reshape only supports 4D tensors\n";
        std::exit(1);
    }
    reshape(d.data(), 4);
}

void NodeBackProp::reshape(int arr[], const int size) {
    if (size != 4) {
        std::cerr << "Reshape only supports 4D tensors\n";
        std::exit(1);
    }
    const long long nt = (long long)arr[0] * arr[1] * arr[2] * arr[3];
    if (nt != total) {
        std::cerr << "Reshape cannot change total size of tensor\n";
        std::cout << "Dimensions for node: " << op_name << "\n";
        std::exit(1);
    }
    for (int i = 0; i < 4; ++i) dim[i] = arr[i];
}

// ============================================================================
// AdamParameter (Engine/engine.cu:126-302)
// ============================================================================
AdamParameter::AdamParameter(str n, int out, int in, int row, int col, double norm)
    : NodeBackProp(n, out, in, row, col, 2), t(1), b1(0.9f), b2(0.999f), epsilon(1e-8f), batch_size(0),
      group_norm((float)norm), weight_decay(0.01f) {
    m = arena_alloc(ARENA_PARAM, total, op_name + " m");
    v = arena_alloc(ARENA_PARAM, total, op_name + " v");
    t_dev = (int32_t*)arena_alloc_bytes(ARENA_WS, sizeof(int32_t), op_name + " t");
    const int32_t one = 1;
    check_cuda(cudaMemcpy(t_dev, &one, sizeof(one), cudaMemcpyHostToDevice), "AdamParameter t");
    // Standard_Weights: uniform(-s, s), s = sqrt(XAVIER / (in*row*col))
    // (Engine/kernels.cu:953-960); the generator is seeded by mle::set_seed
    // when set, else by std::random_device as in the reference.
    uint64_t seed;
    if (g_seeded) {
        seed = g_seed * 0x9E3779B97F4A7C15ull + (++g_param_counter);
    } else {
        std::random_device rd;
        seed = ((uint64_t)rd() << 32) | rd();
    }
    std::mt19937_64 gen(seed);
    const float scale = sqrtf(XAVIER / (float)((long long)in * row * col));
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    std::vector<float> h((size_t)total);
    for (auto& x : h) x = dist(gen) * scale;
    check_cuda(cudaMemcpy(output, h.data(), (size_t)total * sizeof(float), cudaMemcpyHostToDevice),
               "AdamParameter init");
    all_parameters().push_back(this);
}

void AdamParameter::save(std::ofstream& f) const {
    // binary record: u32 name_len, name, i32 total, f32 w[total], m[total], v[total]
    uint32_t name_len = (uint32_t)op_name.size();
    f.write(reinterpret_cast<const char*>(&name_len), sizeof(uint32_t));
    f.write(op_name.data(), name_len);
    const int tot = (int)total;
    f.write(reinterpret_cast<const char*>(&tot), sizeof(int));
    std::vector<float> host((size_t)total);
    const float* srcs[3] = {output, m, v};
    for (const float* src : srcs) {
        check_cuda(cudaStreamSynchronize(g_stream), "save");
        check_cuda(cudaMemcpy(host.data(), src, (size_t)total * sizeof(float), cudaMemcpyDeviceToHost), "save");
        f.write(reinterpret_cast<const char*>(host.data()), total * sizeof(float));
    }
    if (!f) {
        std::cerr << "File write failed saving parameter: " << op_name << "\n";
        std::exit(1);
    }
}

void AdamParameter::load(std::ifstream& f) {
    uint32_t name_len = 0;
    f.read(reinterpret_cast<char*>(&name_len), sizeof(uint32_t));
    std::string loaded(name_len, '\0');
    f.read(&loaded[0], name_len);
    if (!f) {
        std::cerr << "File read failed reading name for: " << op_name << "\n";
        std::exit(1);
    }
    if (loaded != op_name) {
        std::cerr << "Parameter name mismatch: expected '" << op_name << "' but got '" << loaded << "'\n";
        std::exit(1);
    }
    int loaded_total = 0;
    f.read(reinterpret_cast<char*>(&loaded_total), sizeof(int));
    if (loaded_total != total) {
        std::cerr << "Parameter size mismatch for '" << op_name << "': expected " << total << " but loaded "
                  << loaded_total << "\n";
        std::exit(1);
    }
    std::vector<float> host((size_t)total);
    for (float* dst : {output, m, v}) {
        f.read(reinterpret_cast<char*>(host.data()), total * sizeof(float));
        if (!f) {
            std::cerr << "File read failed loading: " << op_name << "\n";
            std::exit(1);
        }
        check_cuda(cudaMemcpy(dst, host.data(), (size_t)total * sizeof(float), cudaMemcpyHostToDevice), "load");
    }
}

void AdamParameter::operator=(const AdamParameter& other) {
    for (int i = 0; i < 4; ++i)
        if (dim[i] != other.dim[i]) {
            std::cout << "Shape Mismatch in equator operator of AdamParameter " << op_name << " and "
                      << other.op_name;
            std::exit(1);
        }
    check(mle_copy(other.output, output, total, st()), op_name + " = " + other.op_name);
}

static mle_param_view view_of(AdamParameter* p) {
    mle_param_view v;
    v.w = p->output;
    v.g = p->grad;
    v.m = p->m;
    v.v = p->v;
    v.n = p->total;
    v.t = p->t_dev;
    v.b1 = p->b1;
    v.b2 = p->b2;
    v.eps = p->epsilon;
    v.weight_decay = p->weight_decay;
    return v;
}

void AdamParameter::update(const float lr, const bool W) {
    if (g_collector) {
        g_collector->update.push_back({this, lr, W});
    } else {
        mle_param_view v = view_of(this);
        check(mle_adam_update(&v, 1, nullptr, 1.0f, lr, W ? 1 : 0, 0, st()), "AdamUpdate of " + op_name);
    }
    t++;
}

void AdamParameter::accumulate_grad(double* global_scale) {
    if (g_collector) {
        g_collector->sumsq.push_back(this);
    } else {
        mle_param_view v = view_of(this);
        check(mle_grad_sumsq(&v, 1, global_scale, 1.0, st()), "SumSquared of " + op_name);
    }
}

void AdamParameter::gradnorm(const double* global_scale) {
    if (g_collector) {
        g_collector->clip.push_back(this);
    } else {
        mle_param_view v = view_of(this);
        check(mle_clip_apply(&v, 1, global_scale, st()), "gradnorm of " + op_name);
    }
}

void AdamParameter::sync_step() {
    int32_t h = 0;
    check_cuda(cudaStreamSynchronize(g_stream), "sync_step");
    check_cuda(cudaMemcpy(&h, t_dev, sizeof(h), cudaMemcpyDeviceToHost), "sync_step");
    t = h;
}

void Dimension(graph X) {
    std::cout << "Dimensions for node: " << X->op_name << " ";
    printf("(%i x %i x %i x %i) \n", X->dim[0], X->dim[1], X->dim[2], X->dim[3]);
}
void Dimension(AdamParameter X) {
    std::cout << "Dimensions for node: " << X.op_name << " ";
    printf("(%i x %i x %i x %i) \n", X.dim[0], X.dim[1], X.dim[2], X.dim[3]);
}
void Zerograd(AdamParameter X) { zero_range(X.grad, X.total); }
void Zerograd(graph X) { zero_range(X->grad, X->total); }

// ============================================================================
// topological sort and drivers (Engine/engine.cu:652-673, 3362-3449)
// ============================================================================
graph_tree topological_sort(const graph& root) {
    std::unordered_set<NodeBackProp*> visited;
    graph_tree result;
    std::function<void(const graph&)> dfs = [&](const graph& node) {
        if (!node || visited.count(node.get())) return;
        visited.insert(node.get());
        for (const auto& in : node->inputs) dfs(in);
        result.push_back(node);
    };
    dfs(root);
    return result;
}

double GraphOperations::GB = 0.0;
bool GraphOperations::calculate_loss = false;
float GraphOperations::loss = 0.0f;

// Runs the given member lambdas with a collector installed and returns the
// distinct parameters in first-touch order; a parameter touched twice in one
// pass (a Linear forwarded twice) is returned twice in separate rounds.
static std::vector<std::vector<AdamParameter*>> rounds_of(const std::vector<AdamParameter*>& list) {
    std::vector<std::vector<AdamParameter*>> rounds;
    std::unordered_map<AdamParameter*, int> seen;
    for (AdamParameter* p : list) {
        const int r = seen[p]++;
        if ((int)rounds.size() <= r) rounds.emplace_back();
        rounds[r].push_back(p);
    }
    return rounds;
}

static void launch_sumsq(const std::vector<AdamParameter*>& ps, double* ws, double scale) {
    std::vector<mle_param_view> v;
    for (auto* p : ps) v.push_back(view_of(p));
    check(mle_grad_sumsq(v.data(), (int)v.size(), ws, scale, st()), "SumSquared (fused)");
}

void GraphOperations::accumulate(double* global_scale) {
    ParamCollector c;
    g_collector = &c;
    for (auto& node : nodes)
        if (node->accumulate) node->accumulate(global_scale);
    g_collector = nullptr;
    // a parameter listed twice adds its square twice, as the reference does
    for (auto& r : rounds_of(c.sumsq)) launch_sumsq(r, global_scale, 1.0);
    check(mle_clip_finalize(global_scale, 1.0, st()), "Sqrt_Scale");
}

void GraphOperations::clipNorm(double* global_scale) {
    ParamCollector c;
    g_collector = &c;
    for (auto& node : nodes)
        if (node->clipnorm) node->clipnorm(global_scale);
    g_collector = nullptr;
    for (auto& r : rounds_of(c.clip)) {
        std::vector<mle_param_view> v;
        for (auto* p : r) v.push_back(view_of(p));
        check(mle_clip_apply(v.data(), (int)v.size(), global_scale, st()), "clipNorm (fused)");
    }
}

void GraphOperations::collect_params(std::vector<AdamParameter*>& out) {
    ParamCollector c;
    g_collector = &c;
    for (auto& node : nodes)
        if (node->accumulate) node->accumulate(nullptr);
    g_collector = nullptr;
    out = c.sumsq;
}

static bool g_fused_optimizer = true;
static bool g_add_norm_fusion = true;
bool mle::add_norm_fusion() { return g_add_norm_fusion; }

extern "C" int mle_set_add_norm_fusion(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    g_add_norm_fusion = enable != 0;
    return MLE_OK;
}

extern "C" int mle_get_add_norm_fusion(void) { return g_add_norm_fusion ? 1 : 0; }

extern "C" int mle_set_fused_optimizer(int enable) {
    if (enable != 0 && enable != 1) return MLE_ERR_ARG;
    g_fused_optimizer = enable != 0;
    return MLE_OK;
}

extern "C" int mle_get_fused_optimizer(void) { return g_fused_optimizer ? 1 : 0; }

void GraphOperations::clip_grad_norm(const float max_norm) {
    if (g_fused_optimizer) {
        // the norm is taken by the next ParameterUpdate's single launch, or
        // by flush_deferred_clip() where that update cannot take it
        clip_max_norm_ = max_norm;
        clip_deferred_ = true;
        clip_pending_ = true;
        return;
    }
    double* ws = clip_workspace();
    check_cuda(cudaMemsetAsync(ws, 0, sizeof(double), g_stream), "clip workspace");
    std::vector<AdamParameter*> ps;
    collect_params(ps);
    for (auto& r : rounds_of(ps)) launch_sumsq(r, ws, (double)grad_prescale_);
    check(mle_clip_finalize(ws, (double)max_norm, st()), "clip finalize");
    clip_pending_ = true;
}

void GraphOperations::flush_deferred_clip() {
    if (!clip_deferred_) return;
    clip_deferred_ = false;
    double* ws = clip_workspace();
    check_cuda(cudaMemsetAsync(ws, 0, sizeof(double), g_stream), "clip workspace");
    std::vector<AdamParameter*> ps;
    collect_params(ps);
    for (auto& r : rounds_of(ps)) launch_sumsq(r, ws, (double)grad_prescale_);
    check(mle_clip_finalize(ws, (double)clip_max_norm_, st()), "clip finalize");
}

// One launch for the norm, the clip, the update and the step counters, when
// the update covers exactly the clipped parameters, each once, with one
// learning rate and rule.  False (nothing launched) when it does not apply.
bool GraphOperations::fused_update(const std::vector<AdamParameter*>& ps, float lr, bool adamw) {
    if (!g_fused_optimizer || ps.empty()) return false;
    std::unordered_set<AdamParameter*> seen(ps.begin(), ps.end());
    if (seen.size() != ps.size()) return false;
    if (clip_deferred_) {
        std::vector<AdamParameter*> cl;
        collect_params(cl);
        if (cl.size() != ps.size()) return false;
        for (auto* p : cl)
            if (!seen.count(p)) return false;
    } else if (clip_pending_) {
        return false;  // a coefficient computed by the separate launches
    }
    std::vector<mle_param_view> v;
    v.reserve(ps.size());
    for (auto* p : ps) v.push_back(view_of(p));
    const bool same = v.size() == fused_views_.size() &&
                      memcmp(v.data(), fused_views_.data(), v.size() * sizeof(mle_param_view)) == 0;
    if (!same) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        check_cuda(cudaStreamIsCapturing(g_stream, &cap), "capture status");
        if (cap != cudaStreamCaptureStatusNone) return false;  // the table is copied from the host
        const int64_t need = mle_clip_adam_ws_bytes((int)v.size());
        if (need > fused_ws_bytes_) {
            fused_ws_ = arena_alloc_bytes(ARENA_WS, need, "optimizer table");
            fused_ws_bytes_ = need;
        }
        check(mle_clip_adam_prepare(v.data(), (int)v.size(), fused_ws_, fused_ws_bytes_, st()), "optimizer table");
        fused_views_ = v;
    }
    const float max_norm = clip_deferred_ ? clip_max_norm_ : 0.0f;
    const bool wb = clip_deferred_ || grad_prescale_ != 1.0f;
    check(mle_clip_adam_run(fused_ws_, max_norm, grad_prescale_, lr, adamw ? 1 : 0, wb ? 1 : 0, st()),
          "norm + clip + AdamWUpdate (one launch)");
    clip_deferred_ = false;
    clip_pending_ = false;
    return true;
}

void GraphOperations::apply_clip() {
    flush_deferred_clip();
    if (!clip_pending_) return;
    clipNorm(clip_workspace());
    clip_pending_ = false;
}

void GraphOperations::ParameterUpdate(const graph& X, const bool show, const float lr, const bool adamw) {
    if (X) nodes = topological_sort(X);
    if (nodes.empty()) {
        printf("Warning... Nodes list is empty and parameter update cannot run.. \n You may have forgotten to "
               "topologically sort \n");
        return;
    }
    ParamCollector c;
    g_collector = &c;
    for (auto& node : nodes)
        if (node->updateParams) node->updateParams(lr, adamw);
    g_collector = nullptr;
    // group by (lr, adamw); repeated parameters go to later rounds
    std::map<std::pair<float, bool>, std::vector<AdamParameter*>> groups;
    for (auto& u : c.update) groups[{u.lr, u.adamw}].push_back(u.p);
    if (groups.size() == 1 && fused_update(groups.begin()->second, groups.begin()->first.first,
                                           groups.begin()->first.second)) {
        if (show)
            for (auto& node : nodes)
                if (node->updateParams) print_head(node->output, node->total, node->op_name);
        return;
    }
    flush_deferred_clip();
    const double* clip = clip_pending_ ? clip_workspace() : nullptr;
    for (auto& g : groups) {
        for (auto& r : rounds_of(g.second)) {
            std::vector<mle_param_view> v;
            for (auto* p : r) v.push_back(view_of(p));
            check(mle_adam_update(v.data(), (int)v.size(), clip, grad_prescale_, g.first.first,
                                  g.first.second ? 1 : 0, (clip || grad_prescale_ != 1.0f) ? 1 : 0, st()),
                  "AdamWUpdate (fused)");
        }
    }
    clip_pending_ = false;
    if (show)
        for (auto& node : nodes)
            if (node->updateParams) print_head(node->output, node->total, node->op_name);
}

void GraphOperations::forward(const graph& X, const bool calc_loss, const bool show, const bool time,
                              const bool check_nan) {
    if (X) nodes = topological_sort(X);
    if (calc_loss) calculate_loss = true;
    if (nodes.empty()) {
        printf("Warning... Nodes list is empty and forward cannot run.. \n You may have forgotten to topologically "
               "sort \n");
        return;
    }
    prepare_fusions(nodes);  // the forward's Add + LayerNorm passes (and the backward's plan)
    for (auto& node : nodes) {
        auto t0 = std::chrono::high_resolution_clock::now();
        if (time) CheckError("Before " + node->op_name + " forward");
        if (node->forward) {
            node->forward();
            if (check_nan) host_nan_check(node->output, node->total, "IsNan of " + node->op_name);
            if (show) {
                Dimension(node);
                print_head(node->output, node->total, node->op_name);
            }
        }
        if (time) {
            CheckError("After " + node->op_name + " forward");
            auto t1 = std::chrono::high_resolution_clock::now();
            std::cout << "Time elapsed for " << node->op_name << " forward: "
                      << std::chrono::duration<double, std::milli>(t1 - t0).count() << "ms \n";
        }
    }
    calculate_loss = false;
}

void GraphOperations::backward(const graph& X, const bool show, const bool time, const bool check_nan) {
    if (X) nodes = topological_sort(X);
    if (nodes.empty()) {
        printf("Warning... Nodes list is empty and bacward cannot run.. \n You may have forgotten to topologically "
               "sort \n");
        return;
    }
    prepare_fusions(nodes);
    for (auto it = nodes.rbegin(); it != nodes.rend(); ++it) {
        auto t0 = std::chrono::high_resolution_clock::now();
        if (time) CheckError("Previous");
        if ((*it)->backward) {
            (*it)->backward();
            if (check_nan) host_nan_check((*it)->grad, (*it)->total, "IsNan of " + (*it)->op_name);
            if (show) print_head((*it)->grad, (*it)->total, (*it)->op_name);
        }
        if (on_backward_done) on_backward_done(it->get());
        if (time) {
            join_param_stream();
            CheckError("After " + (*it)->op_name + " backward");
            auto t1 = std::chrono::high_resolution_clock::now();
            std::cout << "Time elapsed for " << (*it)->op_name << " backward: "
                      << std::chrono::duration<double, std::milli>(t1 - t0).count() << "ms \n";
        }
    }
    join_param_stream();
}

void GraphOperations::zero_grad(const graph& X, const bool show) {
    if (X) nodes = topological_sort(X);
    if (nodes.empty()) {
        printf("Warning... Nodes list is empty and Zero grad cannot run.. \n You may have forgotten to topologically "
               "sort \n");
        return;
    }
    // the skip set must describe this graph: plan its fusions (the same plan
    // backward() makes) before any gradient is left uncleared
    prepare_fusions(nodes);
    struct SkipScope {
        SkipScope() { ++g_skip_depth; }
        ~SkipScope() { --g_skip_depth; }
    } skip;
    ZeroBatch zb;
    for (auto it = nodes.rbegin(); it != nodes.rend(); ++it) {
        if ((*it)->zero_grad) {
            if (show) std::cout << "Zeroing gradient of" + (*it)->op_name + "\n";
            (*it)->zero_grad();
        }
    }
}

void GraphOperations::printParams(const graph& X, const bool show) {
    if (X) nodes = topological_sort(X);
    for (auto& node : nodes)
        if (node->printparams) node->printparams(show);
}

void GraphOperations::printNodes(const graph& X, const int show) {
    for (auto& node : nodes) {
        if (node->zero_grad) {
            std::cout << "Calling Node: " << node->op_name << "\n";
            Dimension(node);
            if (show == 1) print_head(node->output, node->total, node->op_name);
            if (show == 2) print_head(node->grad, node->total, node->op_name);
        }
    }
}

void GraphOperations::clear_graph(const graph& X, const bool show) {
    if (X) nodes = topological_sort(X);
    for (auto& node : nodes)
        if (node->free) {
            if (show) std::cout << "Freeing Node: " << node->op_name << "\n";
            node->free();
        }
    nodes.clear();
}

void GraphOperations::clean_clear_graph(const graph& X, const bool show) {
    if (X) nodes = topological_sort(X);
    for (auto& node : nodes) {
        if (node->free) node->free();
        if (node->serious_free) node->serious_free();
    }
}
