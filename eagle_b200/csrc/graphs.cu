// The graph groups of the eagle-backend/1 seam: capturer (bit 1), captured (2),
// fork (3), conditional (4, with IF/ELSE 13 and SWITCH 14), attribution (5),
// graph (6) and launcher (7), python/src/seam/eagle_backend.h:286-383 of the
// eagle source tree. They let eagle's own captured pipelines (a stream capture in
// thread-local mode, device-evaluated IF / WHILE nodes woven into it, the graph
// instantiated once and replayed) run on this library.
//
// Conditional nodes are evaluated on the device by 1x1 setter kernels of this
// file, so a replay never returns to the host: the guard is
// ``(*count != (baseline ? *baseline : 0)) != negate`` (a null count always
// holds), eagle/conditional/CountGuard.h:11-13; a WHILE keeps a caller-owned
// ``uint32[2] = {remaining, ran}`` cell that its head setter resets every replay
// and its tail setter (the body's last node) advances, with the optional runtime
// trip count and break cell of eagle/conditional/ConditionalGroup.h (LoopTerms).
#include "common.cuh"

#include <cstdlib>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#define EB_API extern "C" __attribute__((visibility("default")))

namespace eb {
namespace {

// ------------------------------------------------------------ device setters

struct Guard {
    const unsigned* count;
    const unsigned* baseline;
    unsigned negate;
};

struct LoopTerms {
    unsigned cap;
    unsigned* counter;  // {remaining, ran}
    const unsigned* limit;
    unsigned* brk;
};

__device__ __forceinline__ bool guardHolds(const Guard& g)
{
    if (g.count == nullptr)
        return true;
    const unsigned base = g.baseline != nullptr ? *g.baseline : 0u;
    return (*g.count != base) != (g.negate != 0u);
}

__global__ void condGuardKernel(cudaGraphConditionalHandle h, Guard g)
{
    cudaGraphSetConditional(h, guardHolds(g) ? 1u : 0u);
}

__global__ void condSwitchKernel(cudaGraphConditionalHandle h, const unsigned* arm)
{
    cudaGraphSetConditional(h, *arm);
}

__global__ void loopHeadKernel(cudaGraphConditionalHandle h, Guard g, LoopTerms t)
{
    t.counter[0] = t.cap;
    t.counter[1] = 0u;
    if (t.brk != nullptr)
        *t.brk = 0u;
    const bool more = t.cap != 0u && (t.limit == nullptr || *t.limit != 0u);
    cudaGraphSetConditional(h, (more && guardHolds(g)) ? 1u : 0u);
}

__global__ void loopTailKernel(cudaGraphConditionalHandle h, Guard g, LoopTerms t)
{
    const unsigned remaining = --t.counter[0];
    const unsigned ran = ++t.counter[1];
    const bool more = remaining != 0u && (t.limit == nullptr || ran < *t.limit) && (t.brk == nullptr || *t.brk == 0u);
    cudaGraphSetConditional(h, (more && guardHolds(g)) ? 1u : 0u);
}

// ------------------------------------------------------------ driver entries

/** Driver entry points for patching instantiated graphs, resolved at the
 *  runtime's version the first time a launcher patches something. */
struct GraphDriver {
    CUresult (*kernelGet)(CUgraphNode, CUDA_KERNEL_NODE_PARAMS*) = nullptr;
    CUresult (*kernelSet)(CUgraphNode, const CUDA_KERNEL_NODE_PARAMS*) = nullptr;
    CUresult (*execKernelSet)(CUgraphExec, CUgraphNode, const CUDA_KERNEL_NODE_PARAMS*) = nullptr;
    CUresult (*paramInfo)(CUfunction, size_t, size_t*, size_t*) = nullptr;
    CUresult (*kernelFunction)(CUfunction*, CUkernel) = nullptr;
    CUresult (*memcpyGet)(CUgraphNode, CUDA_MEMCPY3D*) = nullptr;
    CUresult (*memcpySet)(CUgraphNode, const CUDA_MEMCPY3D*) = nullptr;
    CUresult (*execMemcpySet)(CUgraphExec, CUgraphNode, const CUDA_MEMCPY3D*, CUcontext) = nullptr;
    CUresult (*ctxCurrent)(CUcontext*) = nullptr;
    CUresult (*execUpdate)(CUgraphExec, CUgraph, CUgraphExecUpdateResultInfo*) = nullptr;
    CUresult (*nodeType)(CUgraphNode, CUgraphNodeType*) = nullptr;
};

const GraphDriver& graphDriver()
{
    static GraphDriver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* sym, void** fn) {
            cudaDriverEntryPointQueryResult q{};
            if (cudaGetDriverEntryPointByVersion(sym, fn, CUDART_VERSION, cudaEnableDefault, &q) != cudaSuccess
                || q != cudaDriverEntryPointSuccess)
                *fn = nullptr;
            (void)cudaGetLastError();
        };
        get("cuGraphKernelNodeGetParams", reinterpret_cast<void**>(&d.kernelGet));
        get("cuGraphKernelNodeSetParams", reinterpret_cast<void**>(&d.kernelSet));
        get("cuGraphExecKernelNodeSetParams", reinterpret_cast<void**>(&d.execKernelSet));
        get("cuFuncGetParamInfo", reinterpret_cast<void**>(&d.paramInfo));
        get("cuKernelGetFunction", reinterpret_cast<void**>(&d.kernelFunction));
        get("cuGraphMemcpyNodeGetParams", reinterpret_cast<void**>(&d.memcpyGet));
        get("cuGraphMemcpyNodeSetParams", reinterpret_cast<void**>(&d.memcpySet));
        get("cuGraphExecMemcpyNodeSetParams", reinterpret_cast<void**>(&d.execMemcpySet));
        get("cuCtxGetCurrent", reinterpret_cast<void**>(&d.ctxCurrent));
        get("cuGraphExecUpdate", reinterpret_cast<void**>(&d.execUpdate));
        get("cuGraphNodeGetType", reinterpret_cast<void**>(&d.nodeType));
    });
    return d;
}

template <class F>
F need(F fn, const char* name)
{
    if (fn == nullptr)
        fail(EAGLE_BACKEND_UNAVAILABLE, std::string("eagle_b200: the driver lacks ") + name);
    return fn;
}

// ------------------------------------------------------------------- helpers

/** A node's type, read through the driver (which names every node kind the
 *  driver makes, conditional nodes included). */
CUgraphNodeType nodeType(cudaGraphNode_t node)
{
    CUgraphNodeType t{};
    cuCheck(need(graphDriver().nodeType, "cuGraphNodeGetType")(reinterpret_cast<CUgraphNode>(node), &t),
        "cuGraphNodeGetType");
    return t;
}

/** The device a seam stream belongs to (0: the current device). A stream in
 *  capture answers no device query (the query would invalidate the capture), so
 *  a capturing stream is taken to be on the current device, where its capture
 *  runs. */
int streamDevice(uint64_t stream)
{
    int dev = 0;
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (stream == 0
        || (cudaStreamIsCapturing(reinterpret_cast<cudaStream_t>(stream), &st) == cudaSuccess
            && st != cudaStreamCaptureStatusNone)) {
        cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
        return dev;
    }
    cudaCheck(cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &dev), "cudaStreamGetDevice");
    return dev;
}

/** The graph a stream is capturing into and the nodes its next work depends on. */
struct CaptureTip {
    cudaGraph_t graph = nullptr;
    std::vector<cudaGraphNode_t> deps;
};

CaptureTip captureTip(cudaStream_t s, const std::string& who)
{
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    unsigned long long id = 0;
    CaptureTip tip;
    const cudaGraphNode_t* deps = nullptr;
    const cudaGraphEdgeData* edges = nullptr;
    size_t n = 0;
    cudaCheck(cudaStreamGetCaptureInfo_v3(s, &status, &id, &tip.graph, &deps, &edges, &n),
        "cudaStreamGetCaptureInfo");
    if (status != cudaStreamCaptureStatusActive)
        invalid(who + ": the stream is not capturing");
    tip.deps.assign(deps, deps + n);
    return tip;
}

std::vector<cudaGraphNode_t> graphNodes(cudaGraph_t g)
{
    size_t n = 0;
    cudaCheck(cudaGraphGetNodes(g, nullptr, &n), "cudaGraphGetNodes");
    std::vector<cudaGraphNode_t> nodes(n);
    if (n != 0)
        cudaCheck(cudaGraphGetNodes(g, nodes.data(), &n), "cudaGraphGetNodes");
    nodes.resize(n);
    return nodes;
}

/** A backend-allocated node list (freed by eagle_backend_free). */
void handOut(const std::vector<cudaGraphNode_t>& nodes, uint64_t** out, int64_t* count)
{
    auto* buf = static_cast<uint64_t*>(std::malloc((nodes.empty() ? 1 : nodes.size()) * sizeof(uint64_t)));
    if (buf == nullptr)
        throw std::bad_alloc();
    for (size_t i = 0; i < nodes.size(); ++i)
        buf[i] = reinterpret_cast<uint64_t>(nodes[i]);
    *out = buf;
    *count = int64_t(nodes.size());
}

cudaGraphNode_t addSetter(cudaGraph_t g, const void* fn, void** args, const std::vector<cudaGraphNode_t>& deps)
{
    cudaKernelNodeParams kp{};
    kp.func = const_cast<void*>(fn);
    kp.gridDim = dim3(1, 1, 1);
    kp.blockDim = dim3(1, 1, 1);
    kp.kernelParams = args;
    cudaGraphNode_t node = nullptr;
    cudaCheck(cudaGraphAddKernelNode(&node, g, deps.empty() ? nullptr : deps.data(), deps.size(), &kp),
        "cudaGraphAddKernelNode");
    return node;
}

/** Node types CUDA does not take inside a conditional body (recursing into child
 *  graphs); nullptr when there is none. */
const char* bodyRefusal(cudaGraph_t g, int depth = 0)
{
    for (cudaGraphNode_t node : graphNodes(g)) {
        switch (nodeType(node)) {
        case CU_GRAPH_NODE_TYPE_KERNEL:
        case CU_GRAPH_NODE_TYPE_MEMCPY:
        case CU_GRAPH_NODE_TYPE_MEMSET:
        case CU_GRAPH_NODE_TYPE_EMPTY:
        case CU_GRAPH_NODE_TYPE_CONDITIONAL:
            break;
        case CU_GRAPH_NODE_TYPE_GRAPH: {
            cudaGraph_t inner = nullptr;
            cudaCheck(cudaGraphChildGraphNodeGetGraph(node, &inner), "cudaGraphChildGraphNodeGetGraph");
            if (depth < 16)
                if (const char* found = bodyRefusal(inner, depth + 1))
                    return found;
            break;
        }
        case CU_GRAPH_NODE_TYPE_HOST: return "host";
        case CU_GRAPH_NODE_TYPE_EVENT_RECORD: return "event record";
        case CU_GRAPH_NODE_TYPE_WAIT_EVENT: return "event wait";
        case CU_GRAPH_NODE_TYPE_MEM_ALLOC: return "memory allocation";
        case CU_GRAPH_NODE_TYPE_MEM_FREE: return "memory free";
        default: return "external semaphore or batch memop";
        }
    }
    return nullptr;
}

/** The first node a cloned hand-over graph may not hold: a host-function node
 *  (``host`` set), else a conditional or memory-allocation node; empty if none. */
std::string cloneRefusal(cudaGraph_t g, bool& host, int depth = 0)
{
    std::string found;
    const std::vector<cudaGraphNode_t> nodes = graphNodes(g);
    for (size_t i = 0; i < nodes.size(); ++i) {
        const CUgraphNodeType type = nodeType(nodes[i]);
        std::string what;
        if (type == CU_GRAPH_NODE_TYPE_HOST) {
            host = true;
            return "host-function node #" + std::to_string(i);
        }
        if (type == CU_GRAPH_NODE_TYPE_MEM_ALLOC)
            what = "memory-allocation node #" + std::to_string(i);
        else if (type == CU_GRAPH_NODE_TYPE_MEM_FREE)
            what = "memory-free node #" + std::to_string(i);
        else if (type == CU_GRAPH_NODE_TYPE_CONDITIONAL)
            what = "conditional node #" + std::to_string(i);
        else if (type == CU_GRAPH_NODE_TYPE_GRAPH && depth < 16) {
            cudaGraph_t child = nullptr;
            cudaCheck(cudaGraphChildGraphNodeGetGraph(nodes[i], &child), "cudaGraphChildGraphNodeGetGraph");
            what = cloneRefusal(child, host, depth + 1);
            if (host)
                return what;
        }
        if (!what.empty() && found.empty())
            found = what;
    }
    return found;
}

std::string driverText()
{
    int v = 0;
    (void)cudaDriverGetVersion(&v);
    return "driver " + std::to_string(v / 1000) + "." + std::to_string((v % 1000) / 10);
}

// ------------------------------------------------------------------- handles

enum : uint32_t {
    kCapturer = 0x45424331u,
    kCaptured = 0x45424332u,
    kFork = 0x45424333u,
    kConditional = 0x45424334u,
    kGraph = 0x45424336u,
    kLauncher = 0x45424337u,
};

struct Capturer {
    uint32_t tag = kCapturer;
    int device;
    cudaStream_t stream;
};

struct Captured {
    uint32_t tag = kCaptured;
    int device;
    cudaGraph_t graph;
};

/** Branch streams and the events that order them, all made at create (a capture
 *  in flight on the thread forbids making them later). */
struct Fork {
    uint32_t tag = kFork;
    int device;
    cudaStream_t origin;
    cudaEvent_t forkEvent = nullptr;
    std::vector<cudaStream_t> branches;
    std::vector<cudaEvent_t> joins;
    std::vector<cudaEvent_t> marks;
    size_t marked = 0;
    bool forked = false, joined = false;

    void join()
    {
        if (!forked || joined)
            return;
        for (size_t i = 0; i < branches.size(); ++i)
            cudaCheck(cudaEventRecord(joins[i], branches[i]), "cudaEventRecord");
        for (cudaEvent_t e : joins)
            cudaCheck(cudaStreamWaitEvent(origin, e, 0), "cudaStreamWaitEvent");
        joined = true;
    }
};

struct Conditional {
    uint32_t tag = kConditional;
    int device;
    cudaStream_t origin;
    uint32_t kind;  // EAGLE_BACKEND_COND_*
    Guard guard;
    LoopTerms loop;
    std::vector<cudaStream_t> arms;
    std::vector<cudaGraph_t> armGraphs;
    cudaGraphConditionalHandle handle = 0;
    cudaGraphNode_t setter = nullptr, tail = nullptr;
    unsigned opened = 0;
    bool open = false;

    bool isLoop() const { return kind == EAGLE_BACKEND_COND_WHILE; }

    /** Close every arm capture; a WHILE's tail setter is captured first as the
     *  body's last node. Refuses an arm that launched nothing (an empty body
     *  never completes once it fires). */
    void end()
    {
        if (!open)
            return;
        cudaError_t err = cudaSuccess;
        bool empty = false;
        for (unsigned k = 0; k < opened && err == cudaSuccess; ++k) {
            size_t n = 0;
            err = cudaGraphGetNodes(armGraphs[k], nullptr, &n);
            empty = empty || n == 0;
        }
        if (err == cudaSuccess && !empty && isLoop() && opened == 1) {
            loopTailKernel<<<1, 1, 0, arms[0]>>>(handle, guard, loop);
            err = cudaGetLastError();
            if (err == cudaSuccess) {
                cudaStreamCaptureStatus st{};
                unsigned long long id = 0;
                cudaGraph_t g = nullptr;
                const cudaGraphNode_t* deps = nullptr;
                const cudaGraphEdgeData* edges = nullptr;
                size_t n = 0;
                err = cudaStreamGetCaptureInfo_v3(arms[0], &st, &id, &g, &deps, &edges, &n);
                if (err == cudaSuccess && n == 1)
                    tail = deps[0];
            }
        }
        for (unsigned k = 0; k < opened; ++k) {
            cudaGraph_t out = nullptr;
            const cudaError_t e = cudaStreamEndCapture(arms[k], &out);
            if (err == cudaSuccess)
                err = e;
        }
        open = false;
        opened = 0;
        cudaCheck(err, "eagle_backend_conditional_end");
        if (empty)
            invalid(isLoop() ? "eagle_backend_conditional_end: the loop body launched no work; a WHILE node with an "
                               "empty body never ends, so the step must launch at least one kernel"
                             : "eagle_backend_conditional_end: a guarded arm launched no work; an empty conditional "
                               "body never completes when it fires");
    }
};

struct GraphStore {
    cudaGraph_t graph = nullptr;
    ~GraphStore()
    {
        if (graph != nullptr)
            (void)cudaGraphDestroy(graph);
    }
};

struct Graph {
    uint32_t tag = kGraph;
    int device;
    std::shared_ptr<GraphStore> store;
    std::vector<cudaGraphNode_t> nodes;    // the chain add_node extends
    std::vector<cudaGraphNode_t> kernels;  // kernel nodes gathered from added graphs
    cudaStream_t stream = nullptr;
};

struct KernelSnapshot {
    CUDA_KERNEL_NODE_PARAMS params{};
    std::vector<std::vector<char>> values;  // the captured argument bytes, owned
    std::vector<void*> args;
};

struct Launcher {
    uint32_t tag = kLauncher;
    int device;
    std::shared_ptr<GraphStore> store;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<cudaGraphNode_t> kernels;
    std::unordered_map<cudaGraphNode_t, KernelSnapshot> snapshots;

    const KernelSnapshot& snapshot(cudaGraphNode_t node)
    {
        if (auto it = snapshots.find(node); it != snapshots.end())
            return it->second;
        const GraphDriver& d = graphDriver();
        KernelSnapshot snap;
        cuCheck(need(d.kernelGet, "cuGraphKernelNodeGetParams")(reinterpret_cast<CUgraphNode>(node), &snap.params),
            "reading a kernel node");
        CUfunction f = snap.params.func;
        if (f == nullptr)
            cuCheck(need(d.kernelFunction, "cuKernelGetFunction")(&f, snap.params.kern),
                "resolving a kernel node's function");
        auto info = need(d.paramInfo, "cuFuncGetParamInfo (driver >= 12.4)");
        std::vector<size_t> sizes;
        size_t offset = 0, size = 0;
        while (info(f, sizes.size(), &offset, &size) == CUDA_SUCCESS)
            sizes.push_back(size);
        auto** captured = static_cast<void**>(snap.params.kernelParams);
        if (!sizes.empty() && captured == nullptr)
            invalid("eagle_backend_launcher_set_kernel_params: the node carries packed arguments");
        snap.values.resize(sizes.size());
        snap.args.resize(sizes.size());
        for (size_t i = 0; i < sizes.size(); ++i) {
            const char* v = static_cast<const char*>(captured[i]);
            snap.values[i].assign(v, v + sizes[i]);
            snap.args[i] = snap.values[i].data();
        }
        return snapshots.emplace(node, std::move(snap)).first->second;
    }
};

template <class T>
T* live(void* h, uint32_t tag, const char* who)
{
    auto* p = static_cast<T*>(h);
    if (p == nullptr || p->tag != tag)
        fail(EAGLE_BACKEND_BAD_HANDLE, std::string(who) + ": not a live handle");
    return p;
}

template <class T>
void retire(T* p)
{
    p->tag = 0;
    delete p;
}

void nonNull(const void* p, const char* who)
{
    if (p == nullptr)
        invalid(std::string(who) + ": null output pointer");
}

}  // namespace
}  // namespace eb

using namespace eb;

// ---- capturer --------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_capturer_create(const struct eagle_backend_capturer_desc* desc,
    eagle_backend_capturer* out)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0, "eagle_backend_capturer_create");
        nonNull(out, "eagle_backend_capturer_create");
        requireDevice();
        const int dev = d.device >= 0 ? resolveDevice(d.device, 0) : streamDevice(d.stream);
        *out = reinterpret_cast<eagle_backend_capturer>(new Capturer{kCapturer, dev,
            reinterpret_cast<cudaStream_t>(d.stream)});
    });
}

EB_API eagle_backend_status eagle_backend_capturer_begin(eagle_backend_capturer h)
{
    return guarded([&] {
        auto* c = live<Capturer>(h, kCapturer, "eagle_backend_capturer_begin");
        DeviceScope scope(c->device);
        cudaCheck(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    });
}

EB_API eagle_backend_status eagle_backend_capturer_end(eagle_backend_capturer h, eagle_backend_captured* out)
{
    return guarded([&] {
        auto* c = live<Capturer>(h, kCapturer, "eagle_backend_capturer_end");
        nonNull(out, "eagle_backend_capturer_end");
        DeviceScope scope(c->device);
        cudaGraph_t g = nullptr;
        cudaCheck(cudaStreamEndCapture(c->stream, &g), "cudaStreamEndCapture");
        *out = reinterpret_cast<eagle_backend_captured>(new Captured{kCaptured, c->device, g});
    });
}

EB_API eagle_backend_status eagle_backend_capturer_graph(eagle_backend_capturer h, uint64_t* graph)
{
    return guarded([&] {
        auto* c = live<Capturer>(h, kCapturer, "eagle_backend_capturer_graph");
        nonNull(graph, "eagle_backend_capturer_graph");
        DeviceScope scope(c->device);
        cudaStreamCaptureStatus st{};
        unsigned long long id = 0;
        cudaGraph_t g = nullptr;
        const cudaGraphNode_t* deps = nullptr;
        const cudaGraphEdgeData* edges = nullptr;
        size_t n = 0;
        cudaCheck(cudaStreamGetCaptureInfo_v3(c->stream, &st, &id, &g, &deps, &edges, &n),
            "cudaStreamGetCaptureInfo");
        *graph = st == cudaStreamCaptureStatusActive ? reinterpret_cast<uint64_t>(g) : 0;
    });
}

EB_API void eagle_backend_capturer_release(eagle_backend_capturer h)
{
    auto* c = reinterpret_cast<Capturer*>(h);
    if (c != nullptr && c->tag == kCapturer)
        retire(c);
}

// ---- captured --------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_captured_is_valid(eagle_backend_captured h, int32_t* valid)
{
    return guarded([&] {
        auto* c = live<Captured>(h, kCaptured, "eagle_backend_captured_is_valid");
        nonNull(valid, "eagle_backend_captured_is_valid");
        *valid = c->graph != nullptr ? 1 : 0;
    });
}

EB_API void eagle_backend_captured_release(eagle_backend_captured h)
{
    auto* c = reinterpret_cast<Captured*>(h);
    if (c == nullptr || c->tag != kCaptured)
        return;
    if (c->graph != nullptr)
        (void)cudaGraphDestroy(c->graph);
    retire(c);
}

// ---- fork ------------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_fork_create(const struct eagle_backend_fork_desc* desc,
    eagle_backend_fork* out)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0, "eagle_backend_fork_create");
        nonNull(out, "eagle_backend_fork_create");
        requireDevice();
        if (d.branch_count > 4096 || d.wait_count > 65536)
            invalid("eagle_backend_fork_create: branch_count <= 4096 and wait_count <= 65536");
        const int dev = d.device >= 0 ? resolveDevice(d.device, 0) : streamDevice(d.origin);
        DeviceScope scope(dev);
        auto f = std::make_unique<Fork>();
        f->device = dev;
        f->origin = reinterpret_cast<cudaStream_t>(d.origin);
        auto cleanup = [&] {
            for (cudaStream_t s : f->branches)
                (void)cudaStreamDestroy(s);
            for (cudaEvent_t e : f->joins)
                (void)cudaEventDestroy(e);
            for (cudaEvent_t e : f->marks)
                (void)cudaEventDestroy(e);
            if (f->forkEvent != nullptr)
                (void)cudaEventDestroy(f->forkEvent);
        };
        try {
            cudaCheck(cudaEventCreateWithFlags(&f->forkEvent, cudaEventDisableTiming), "cudaEventCreateWithFlags");
            for (uint64_t i = 0; i < d.branch_count; ++i) {
                cudaStream_t s = nullptr;
                cudaCheck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
                f->branches.push_back(s);
                cudaEvent_t e = nullptr;
                cudaCheck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreateWithFlags");
                f->joins.push_back(e);
            }
            for (uint64_t i = 0; i < d.wait_count; ++i) {
                cudaEvent_t e = nullptr;
                cudaCheck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreateWithFlags");
                f->marks.push_back(e);
            }
        } catch (...) {
            cleanup();
            throw;
        }
        *out = reinterpret_cast<eagle_backend_fork>(f.release());
    });
}

EB_API eagle_backend_status eagle_backend_fork_fork(eagle_backend_fork h)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_fork");
        if (f->forked)
            return;
        DeviceScope scope(f->device);
        cudaCheck(cudaEventRecord(f->forkEvent, f->origin), "cudaEventRecord");
        for (cudaStream_t b : f->branches)
            cudaCheck(cudaStreamWaitEvent(b, f->forkEvent, 0), "cudaStreamWaitEvent");
        f->forked = true;
        f->joined = false;
    });
}

EB_API eagle_backend_status eagle_backend_fork_join(eagle_backend_fork h)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_join");
        DeviceScope scope(f->device);
        f->join();
    });
}

EB_API eagle_backend_status eagle_backend_fork_branch(eagle_backend_fork h, uint64_t i, uint64_t* stream)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_branch");
        nonNull(stream, "eagle_backend_fork_branch");
        if (i >= f->branches.size())
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_fork_branch: branch " + std::to_string(i) + " of "
                + std::to_string(f->branches.size()));
        *stream = reinterpret_cast<uint64_t>(f->branches[size_t(i)]);
    });
}

EB_API eagle_backend_status eagle_backend_fork_origin(eagle_backend_fork h, uint64_t* stream)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_origin");
        nonNull(stream, "eagle_backend_fork_origin");
        *stream = reinterpret_cast<uint64_t>(f->origin);
    });
}

EB_API eagle_backend_status eagle_backend_fork_forked(eagle_backend_fork h, int32_t* forked)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_forked");
        nonNull(forked, "eagle_backend_fork_forked");
        *forked = (f->forked && !f->joined) ? 1 : 0;
    });
}

EB_API eagle_backend_status eagle_backend_fork_size(eagle_backend_fork h, uint64_t* n)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_size");
        nonNull(n, "eagle_backend_fork_size");
        *n = f->branches.size();
    });
}

EB_API eagle_backend_status eagle_backend_fork_mark(eagle_backend_fork h, uint64_t producer, uint64_t* mark)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_mark");
        nonNull(mark, "eagle_backend_fork_mark");
        if (f->marked >= f->marks.size())
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_fork_mark: every pre-made mark is used (create the fork with a "
                                      "larger wait_count)");
        if (producer >= f->branches.size())
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_fork_mark: branch index out of range");
        DeviceScope scope(f->device);
        cudaCheck(cudaEventRecord(f->marks[f->marked], f->branches[size_t(producer)]), "cudaEventRecord");
        *mark = f->marked++;
    });
}

EB_API eagle_backend_status eagle_backend_fork_wait(eagle_backend_fork h, uint64_t waiter, uint64_t mark)
{
    return guarded([&] {
        auto* f = live<Fork>(h, kFork, "eagle_backend_fork_wait");
        if (waiter >= f->branches.size() || mark >= f->marked)
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_fork_wait: branch or mark index out of range");
        DeviceScope scope(f->device);
        cudaCheck(cudaStreamWaitEvent(f->branches[size_t(waiter)], f->marks[size_t(mark)], 0), "cudaStreamWaitEvent");
    });
}

EB_API void eagle_backend_fork_release(eagle_backend_fork h)
{
    auto* f = reinterpret_cast<Fork*>(h);
    if (f == nullptr || f->tag != kFork)
        return;
    int prev = -1;
    if (cudaGetDevice(&prev) == cudaSuccess)
        (void)cudaSetDevice(f->device);
    try {
        f->join();
    } catch (...) {
        // a failed join is already reported by the capture it breaks
    }
    for (cudaStream_t s : f->branches)
        (void)cudaStreamDestroy(s);
    for (cudaEvent_t e : f->joins)
        (void)cudaEventDestroy(e);
    for (cudaEvent_t e : f->marks)
        (void)cudaEventDestroy(e);
    (void)cudaEventDestroy(f->forkEvent);
    (void)cudaGetLastError();
    if (prev >= 0)
        (void)cudaSetDevice(prev);
    retire(f);
}

// ---- conditional -------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_conditional_create(const struct eagle_backend_conditional_desc* desc,
    eagle_backend_conditional* out)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0, "eagle_backend_conditional_create");
        nonNull(out, "eagle_backend_conditional_create");
        requireDevice();
        uint32_t kind = d.counter_ptr != 0 ? EAGLE_BACKEND_COND_WHILE : EAGLE_BACKEND_COND_IF;
        if (d.kind > EAGLE_BACKEND_COND_SWITCH)
            unsupported("eagle_backend_conditional_create: unknown kind " + std::to_string(d.kind));
        if (d.kind != 0)
            kind = d.kind;
        const uint32_t own = kind == EAGLE_BACKEND_COND_IF_ELSE ? 2u : 1u;
        const uint32_t arms = d.arms == 0 ? own : d.arms;
        if (kind != EAGLE_BACKEND_COND_SWITCH && arms != own)
            invalid("eagle_backend_conditional_create: IF and WHILE take one arm, IF/ELSE two; only SWITCH takes n");
        if (arms > 1024)
            invalid("eagle_backend_conditional_create: at most 1024 arms");
        if (kind == EAGLE_BACKEND_COND_SWITCH && d.count_ptr == 0)
            invalid("eagle_backend_conditional_create: a SWITCH needs the device arm-index cell (count_ptr)");
        if (kind == EAGLE_BACKEND_COND_WHILE) {
            if (d.counter_ptr == 0)
                invalid("eagle_backend_conditional_create: a WHILE needs a device {remaining, ran} cell (counter_ptr)");
            if (d.loop_cap == 0)
                invalid("eagle_backend_conditional_create: loop_cap must be >= 1");
        }
        if (kind == EAGLE_BACKEND_COND_IF_ELSE || kind == EAGLE_BACKEND_COND_SWITCH) {
            int v = 0;
            if (cudaDriverGetVersion(&v) != cudaSuccess || v < 12080)
                fail(EAGLE_BACKEND_UNAVAILABLE, "eagle_backend_conditional_create: IF/ELSE and SWITCH nodes need a "
                                                "driver >= 12.8 (" + driverText() + ")");
        }
        const uint64_t firstPtr = d.count_ptr != 0 ? d.count_ptr : d.counter_ptr;
        const int dev = d.device >= 0 ? resolveDevice(d.device, 0)
            : d.origin != 0 ? streamDevice(d.origin) : resolveDevice(-1, firstPtr);
        DeviceScope scope(dev);
        auto c = std::make_unique<Conditional>();
        c->device = dev;
        c->origin = reinterpret_cast<cudaStream_t>(d.origin);
        c->kind = kind;
        c->guard = Guard{reinterpret_cast<const unsigned*>(d.count_ptr),
            reinterpret_cast<const unsigned*>(d.baseline_ptr), d.negate};
        c->loop = LoopTerms{d.loop_cap, reinterpret_cast<unsigned*>(d.counter_ptr),
            reinterpret_cast<const unsigned*>(d.limit_ptr), reinterpret_cast<unsigned*>(d.brk_ptr)};
        try {
            for (uint32_t k = 0; k < arms; ++k) {
                cudaStream_t s = nullptr;
                cudaCheck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
                c->arms.push_back(s);
            }
        } catch (...) {
            for (cudaStream_t s : c->arms)
                (void)cudaStreamDestroy(s);
            throw;
        }
        c->armGraphs.assign(arms, nullptr);
        *out = reinterpret_cast<eagle_backend_conditional>(c.release());
    });
}

EB_API eagle_backend_status eagle_backend_conditional_begin(eagle_backend_conditional h, uint64_t* body_stream)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_begin");
        nonNull(body_stream, "eagle_backend_conditional_begin");
        if (c->open)
            invalid("eagle_backend_conditional_begin: already begun");
        DeviceScope scope(c->device);
        const CaptureTip tip = captureTip(c->origin, "eagle_backend_conditional_begin");
        cudaCheck(cudaGraphConditionalHandleCreate(&c->handle, tip.graph, 0, 0), "cudaGraphConditionalHandleCreate");
        cudaGraphConditionalNodeType type = cudaGraphCondTypeIf;
        if (c->kind == EAGLE_BACKEND_COND_WHILE) {
            void* args[] = {&c->handle, &c->guard, &c->loop};
            c->setter = addSetter(tip.graph, reinterpret_cast<const void*>(&loopHeadKernel), args, tip.deps);
            type = cudaGraphCondTypeWhile;
        } else if (c->kind == EAGLE_BACKEND_COND_SWITCH) {
            const unsigned* arm = c->guard.count;
            void* args[] = {&c->handle, &arm};
            c->setter = addSetter(tip.graph, reinterpret_cast<const void*>(&condSwitchKernel), args, tip.deps);
            type = cudaGraphCondTypeSwitch;
        } else {
            void* args[] = {&c->handle, &c->guard};
            c->setter = addSetter(tip.graph, reinterpret_cast<const void*>(&condGuardKernel), args, tip.deps);
        }
        cudaGraphNodeParams cp{};
        cp.type = cudaGraphNodeTypeConditional;
        cp.conditional.handle = c->handle;
        cp.conditional.type = type;
        cp.conditional.size = unsigned(c->arms.size());
        cudaGraphNode_t node = nullptr;
        cudaCheck(cudaGraphAddNode(&node, tip.graph, &c->setter, 1, &cp), "cudaGraphAddNode (conditional)");
        cudaCheck(cudaStreamUpdateCaptureDependencies(c->origin, &node, 1, cudaStreamSetCaptureDependencies),
            "cudaStreamUpdateCaptureDependencies");
        for (size_t k = 0; k < c->arms.size(); ++k)
            c->armGraphs[k] = cp.conditional.phGraph_out[k];
        c->open = true;
        for (size_t k = 0; k < c->arms.size(); ++k) {
            cudaCheck(cudaStreamBeginCaptureToGraph(c->arms[k], c->armGraphs[k], nullptr, nullptr, 0,
                          cudaStreamCaptureModeThreadLocal),
                "cudaStreamBeginCaptureToGraph");
            ++c->opened;
        }
        *body_stream = reinterpret_cast<uint64_t>(c->arms[0]);
    });
}

EB_API eagle_backend_status eagle_backend_conditional_body_stream(eagle_backend_conditional h, uint64_t* body_stream)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_body_stream");
        nonNull(body_stream, "eagle_backend_conditional_body_stream");
        *body_stream = reinterpret_cast<uint64_t>(c->arms[0]);
    });
}

EB_API eagle_backend_status eagle_backend_conditional_is_loop(eagle_backend_conditional h, int32_t* is_loop)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_is_loop");
        nonNull(is_loop, "eagle_backend_conditional_is_loop");
        *is_loop = c->isLoop() ? 1 : 0;
    });
}

EB_API eagle_backend_status eagle_backend_conditional_end(eagle_backend_conditional h)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_end");
        DeviceScope scope(c->device);
        c->end();
    });
}

EB_API eagle_backend_status eagle_backend_conditional_arm_stream(eagle_backend_conditional h, uint64_t k,
    uint64_t* stream)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_arm_stream");
        nonNull(stream, "eagle_backend_conditional_arm_stream");
        if (k >= c->arms.size())
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_conditional_arm_stream: arm index out of range");
        *stream = reinterpret_cast<uint64_t>(c->arms[size_t(k)]);
    });
}

EB_API eagle_backend_status eagle_backend_conditional_nodes(eagle_backend_conditional h, int64_t which,
    uint64_t** nodes, int64_t* count)
{
    return guarded([&] {
        auto* c = live<Conditional>(h, kConditional, "eagle_backend_conditional_nodes");
        nonNull(nodes, "eagle_backend_conditional_nodes");
        nonNull(count, "eagle_backend_conditional_nodes");
        if (which < -1 || which >= int64_t(c->arms.size()))
            fail(EAGLE_BACKEND_INDEX, "eagle_backend_conditional_nodes: arm index out of range");
        DeviceScope scope(c->device);
        std::vector<cudaGraphNode_t> found;
        if (which < 0) {
            if (c->setter != nullptr)
                found.push_back(c->setter);
            if (c->tail != nullptr)
                found.push_back(c->tail);
        } else if (c->armGraphs[size_t(which)] != nullptr) {
            found = graphNodes(c->armGraphs[size_t(which)]);
        }
        handOut(found, nodes, count);
    });
}

EB_API void eagle_backend_conditional_release(eagle_backend_conditional h)
{
    auto* c = reinterpret_cast<Conditional*>(h);
    if (c == nullptr || c->tag != kConditional)
        return;
    int prev = -1;
    if (cudaGetDevice(&prev) == cudaSuccess)
        (void)cudaSetDevice(c->device);
    try {
        c->end();
    } catch (...) {
        // already reported by the capture that is about to fail
    }
    for (cudaStream_t s : c->arms)
        (void)cudaStreamDestroy(s);
    (void)cudaGetLastError();
    if (prev >= 0)
        (void)cudaSetDevice(prev);
    retire(c);
}

// ---- attribution ---------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_capture_snapshot_nodes(uint64_t stream, uint64_t** nodes, int64_t* count)
{
    return guarded([&] {
        nonNull(nodes, "eagle_backend_capture_snapshot_nodes");
        nonNull(count, "eagle_backend_capture_snapshot_nodes");
        requireDevice();
        DeviceScope scope(streamDevice(stream));
        const CaptureTip tip = captureTip(seamStream(stream), "eagle_backend_capture_snapshot_nodes");
        handOut(graphNodes(tip.graph), nodes, count);
    });
}

EB_API eagle_backend_status eagle_backend_is_node_toggleable(uint64_t node, int32_t* toggleable)
{
    return guarded([&] {
        nonNull(toggleable, "eagle_backend_is_node_toggleable");
        if (node == 0)
            invalid("eagle_backend_is_node_toggleable: null node");
        const CUgraphNodeType type = nodeType(reinterpret_cast<cudaGraphNode_t>(node));
        *toggleable = (type == CU_GRAPH_NODE_TYPE_KERNEL || type == CU_GRAPH_NODE_TYPE_MEMCPY
                          || type == CU_GRAPH_NODE_TYPE_MEMSET)
            ? 1
            : 0;
    });
}

EB_API eagle_backend_status eagle_backend_capture_add_child(uint64_t stream, uint64_t child, int32_t conditional_body)
{
    return guarded([&] {
        if (child == 0)
            invalid("eagle_backend_capture_add_child: null graph");
        requireDevice();
        DeviceScope scope(streamDevice(stream));
        auto g = reinterpret_cast<cudaGraph_t>(child);
        if (conditional_body != 0)
            if (const char* type = bodyRefusal(g))
                invalid(std::string("eagle_backend_capture_add_child: the graph holds a node of type '") + type
                    + "', which CUDA does not allow inside a conditional or loop body");
        const cudaStream_t s = seamStream(stream);
        const CaptureTip tip = captureTip(s, "eagle_backend_capture_add_child");
        cudaGraphNode_t node = nullptr;
        cudaCheck(cudaGraphAddChildGraphNode(&node, tip.graph, tip.deps.empty() ? nullptr : tip.deps.data(),
                      tip.deps.size(), g),
            "cudaGraphAddChildGraphNode");
        cudaCheck(cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies),
            "cudaStreamUpdateCaptureDependencies");
    });
}

// ---- graph ---------------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_graph_create(const struct eagle_backend_graph_desc* desc,
    eagle_backend_graph* out)
{
    return guarded([&] {
        const auto d = readDesc(desc, 0, "eagle_backend_graph_create");
        nonNull(out, "eagle_backend_graph_create");
        requireDevice();
        const int dev = resolveDevice(d.device, 0);
        DeviceScope scope(dev);
        auto g = std::make_unique<Graph>();
        g->device = dev;
        g->store = std::make_shared<GraphStore>();
        cudaCheck(cudaGraphCreate(&g->store->graph, 0), "cudaGraphCreate");
        cudaGraphNode_t root = nullptr;
        cudaCheck(cudaGraphAddEmptyNode(&root, g->store->graph, nullptr, 0), "cudaGraphAddEmptyNode");
        g->nodes.push_back(root);
        *out = reinterpret_cast<eagle_backend_graph>(g.release());
    });
}

EB_API eagle_backend_status eagle_backend_graph_from_captured(eagle_backend_captured captured,
    eagle_backend_graph* out)
{
    return guarded([&] {
        auto* c = live<Captured>(captured, kCaptured, "eagle_backend_graph_from_captured");
        nonNull(out, "eagle_backend_graph_from_captured");
        if (c->graph == nullptr)
            invalid("eagle_backend_graph_from_captured: the captured graph is empty (a capture never begun, already "
                    "consumed, or ended in a failed state)");
        auto g = std::make_unique<Graph>();
        g->device = c->device;
        g->store = std::make_shared<GraphStore>();
        g->store->graph = c->graph;
        c->graph = nullptr;
        retire(c);
        *out = reinterpret_cast<eagle_backend_graph>(g.release());
    });
}

EB_API eagle_backend_status eagle_backend_graph_stream(eagle_backend_graph h, uint64_t stream)
{
    return guarded([&] {
        live<Graph>(h, kGraph, "eagle_backend_graph_stream")->stream = reinterpret_cast<cudaStream_t>(stream);
    });
}

EB_API eagle_backend_status eagle_backend_graph_add_node(eagle_backend_graph h, eagle_backend_captured captured)
{
    return guarded([&] {
        auto* g = live<Graph>(h, kGraph, "eagle_backend_graph_add_node");
        auto* c = live<Captured>(captured, kCaptured, "eagle_backend_graph_add_node");
        if (c->graph == nullptr)
            invalid("eagle_backend_graph_add_node: the captured graph is empty");
        DeviceScope scope(g->device);
        cudaGraphNode_t node = nullptr;
        cudaGraphNode_t* dep = g->nodes.empty() ? nullptr : &g->nodes.back();
        cudaCheck(cudaGraphAddChildGraphNode(&node, g->store->graph, dep, dep ? 1 : 0, c->graph),
            "cudaGraphAddChildGraphNode");
        g->nodes.push_back(node);
        cudaGraph_t embedded = nullptr;
        cudaCheck(cudaGraphChildGraphNodeGetGraph(node, &embedded), "cudaGraphChildGraphNodeGetGraph");
        for (cudaGraphNode_t inner : graphNodes(embedded))
            if (nodeType(inner) == CU_GRAPH_NODE_TYPE_KERNEL)
                g->kernels.push_back(inner);
        (void)cudaGraphDestroy(c->graph);  // the child node holds its own copy
        c->graph = nullptr;
        retire(c);
    });
}

EB_API eagle_backend_status eagle_backend_graph_launcher(eagle_backend_graph h, eagle_backend_launcher* out)
{
    return guarded([&] {
        auto* g = live<Graph>(h, kGraph, "eagle_backend_graph_launcher");
        nonNull(out, "eagle_backend_graph_launcher");
        DeviceScope scope(g->device);
        (void)cudaGetLastError();
        auto l = std::make_unique<Launcher>();
        l->device = g->device;
        l->store = g->store;
        l->stream = g->stream;
        l->kernels = g->kernels;
        cudaCheck(cudaGraphInstantiate(&l->exec, g->store->graph, 0), "cudaGraphInstantiate");
        *out = reinterpret_cast<eagle_backend_launcher>(l.release());
    });
}

EB_API eagle_backend_status eagle_backend_graph_last_node(eagle_backend_graph h, int64_t* index)
{
    return guarded([&] {
        auto* g = live<Graph>(h, kGraph, "eagle_backend_graph_last_node");
        nonNull(index, "eagle_backend_graph_last_node");
        *index = int64_t(g->nodes.size()) - 1;
    });
}

EB_API void eagle_backend_graph_release(eagle_backend_graph h)
{
    auto* g = reinterpret_cast<Graph*>(h);
    if (g != nullptr && g->tag == kGraph)
        retire(g);
}

// ---- launcher --------------------------------------------------------------------------

EB_API eagle_backend_status eagle_backend_launcher_launch(eagle_backend_launcher h)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_launch");
        DeviceScope scope(l->device);
        cudaCheck(cudaGraphLaunch(l->exec, l->stream), "cudaGraphLaunch");
    });
}

EB_API eagle_backend_status eagle_backend_launcher_synchronize(eagle_backend_launcher h)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_synchronize");
        DeviceScope scope(l->device);
        cudaCheck(cudaStreamSynchronize(l->stream), "cudaStreamSynchronize");
    });
}

EB_API eagle_backend_status eagle_backend_launcher_stream(eagle_backend_launcher h, uint64_t stream)
{
    return guarded([&] {
        live<Launcher>(h, kLauncher, "eagle_backend_launcher_stream")->stream = reinterpret_cast<cudaStream_t>(stream);
    });
}

EB_API eagle_backend_status eagle_backend_launcher_set_logical_size(eagle_backend_launcher h, int64_t logical_size)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_set_logical_size");
        if (logical_size < 0)
            invalid("eagle_backend_launcher_set_logical_size: negative size");
        if (logical_size == 0)
            return;
        DeviceScope scope(l->device);
        const GraphDriver& d = graphDriver();
        for (cudaGraphNode_t node : l->kernels) {
            CUDA_KERNEL_NODE_PARAMS p{};
            cuCheck(need(d.kernelGet, "cuGraphKernelNodeGetParams")(reinterpret_cast<CUgraphNode>(node), &p),
                "reading a kernel node");
            const int64_t block = p.blockDimX == 0 ? 1 : int64_t(p.blockDimX);
            const int64_t grid = (logical_size + block - 1) / block;
            if (grid > 0x7fffffff)
                invalid("eagle_backend_launcher_set_logical_size: the grid would exceed 2^31 - 1 blocks");
            p.gridDimX = unsigned(grid);
            p.gridDimY = p.gridDimZ = 1;
            p.blockDimX = unsigned(block);
            p.blockDimY = p.blockDimZ = 1;
            cuCheck(need(d.execKernelSet, "cuGraphExecKernelNodeSetParams")(reinterpret_cast<CUgraphExec>(l->exec),
                        reinterpret_cast<CUgraphNode>(node), &p),
                "re-gridding a kernel node");
        }
    });
}

EB_API eagle_backend_status eagle_backend_launcher_kernel_node_count(eagle_backend_launcher h, int64_t* count)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_kernel_node_count");
        nonNull(count, "eagle_backend_launcher_kernel_node_count");
        *count = int64_t(l->kernels.size());
    });
}

EB_API eagle_backend_status eagle_backend_launcher_set_node_enabled(eagle_backend_launcher h, uint64_t node,
    int32_t enabled)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_set_node_enabled");
        if (node == 0)
            invalid("eagle_backend_launcher_set_node_enabled: null node");
        DeviceScope scope(l->device);
        cudaCheck(cudaGraphNodeSetEnabled(l->exec, reinterpret_cast<cudaGraphNode_t>(node), enabled != 0 ? 1u : 0u),
            "cudaGraphNodeSetEnabled");
    });
}

EB_API eagle_backend_status eagle_backend_launcher_set_kernel_params(eagle_backend_launcher h, uint64_t node,
    const uint64_t* params, int64_t n)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_set_kernel_params");
        if (n < 0 || (n > 0 && params == nullptr) || node == 0)
            invalid("eagle_backend_launcher_set_kernel_params: bad params");
        DeviceScope scope(l->device);
        const KernelSnapshot& snap = l->snapshot(reinterpret_cast<cudaGraphNode_t>(node));
        if (size_t(n) > snap.args.size())
            invalid("eagle_backend_launcher_set_kernel_params: " + std::to_string(n) + " arguments for a kernel taking "
                + std::to_string(snap.args.size()));
        std::vector<void*> args(snap.args);
        for (int64_t i = 0; i < n; ++i)
            if (params[i] != 0)
                args[size_t(i)] = reinterpret_cast<void*>(params[i]);
        CUDA_KERNEL_NODE_PARAMS p = snap.params;
        p.kernelParams = args.data();
        p.extra = nullptr;
        const GraphDriver& d = graphDriver();
        cuCheck(need(d.execKernelSet, "cuGraphExecKernelNodeSetParams")(reinterpret_cast<CUgraphExec>(l->exec),
                    reinterpret_cast<CUgraphNode>(node), &p),
            "patching a kernel node's arguments");
        cuCheck(need(d.kernelSet, "cuGraphKernelNodeSetParams")(reinterpret_cast<CUgraphNode>(node), &p),
            "patching a kernel node's arguments in the source graph");
    });
}

EB_API eagle_backend_status eagle_backend_launcher_set_memcpy_source(eagle_backend_launcher h, uint64_t node,
    uint64_t src)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_set_memcpy_source");
        if (node == 0)
            invalid("eagle_backend_launcher_set_memcpy_source: null node");
        DeviceScope scope(l->device);
        const GraphDriver& d = graphDriver();
        CUDA_MEMCPY3D p{};
        cuCheck(need(d.memcpyGet, "cuGraphMemcpyNodeGetParams")(reinterpret_cast<CUgraphNode>(node), &p),
            "reading a memcpy node");
        if (p.srcMemoryType == CU_MEMORYTYPE_HOST)
            p.srcHost = reinterpret_cast<const void*>(src);
        else if (p.srcMemoryType == CU_MEMORYTYPE_DEVICE || p.srcMemoryType == CU_MEMORYTYPE_UNIFIED)
            p.srcDevice = CUdeviceptr(src);
        else
            invalid("eagle_backend_launcher_set_memcpy_source: the node copies from an array");
        CUcontext ctx = nullptr;
        cuCheck(need(d.ctxCurrent, "cuCtxGetCurrent")(&ctx), "reading the current context");
        cuCheck(need(d.execMemcpySet, "cuGraphExecMemcpyNodeSetParams")(reinterpret_cast<CUgraphExec>(l->exec),
                    reinterpret_cast<CUgraphNode>(node), &p, ctx),
            "re-pointing a memcpy node");
        cuCheck(need(d.memcpySet, "cuGraphMemcpyNodeSetParams")(reinterpret_cast<CUgraphNode>(node), &p),
            "re-pointing a memcpy node in the source graph");
    });
}

EB_API eagle_backend_status eagle_backend_launcher_exec_update(eagle_backend_launcher h,
    eagle_backend_captured captured, int32_t* accepted)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_exec_update");
        auto* c = live<Captured>(captured, kCaptured, "eagle_backend_launcher_exec_update");
        nonNull(accepted, "eagle_backend_launcher_exec_update");
        if (c->graph == nullptr)
            invalid("eagle_backend_launcher_exec_update: the captured graph is empty");
        DeviceScope scope(l->device);
        CUgraphExecUpdateResultInfo info{};
        const CUresult r = need(graphDriver().execUpdate, "cuGraphExecUpdate")(reinterpret_cast<CUgraphExec>(l->exec),
            reinterpret_cast<CUgraph>(c->graph), &info);
        if (r == CUDA_ERROR_GRAPH_EXEC_UPDATE_FAILURE) {
            *accepted = 0;
            return;
        }
        cuCheck(r, "updating the exec graph");
        *accepted = 1;
    });
}

EB_API eagle_backend_status eagle_backend_launcher_clone_graph(eagle_backend_launcher h, uint64_t* graph)
{
    return guarded([&] {
        auto* l = live<Launcher>(h, kLauncher, "eagle_backend_launcher_clone_graph");
        nonNull(graph, "eagle_backend_launcher_clone_graph");
        DeviceScope scope(l->device);
        bool host = false;
        const std::string refused = cloneRefusal(l->store->graph, host);
        if (!refused.empty())
            unsupported("eagle_backend_launcher_clone_graph: the graph holds a " + refused
                + (host ? ", which a handed-over graph may not hold" : ", which CUDA does not take as a child graph")
                + " (" + driverText() + ")");
        cudaGraph_t clone = nullptr;
        cudaCheck(cudaGraphClone(&clone, l->store->graph), "cudaGraphClone");
        *graph = reinterpret_cast<uint64_t>(clone);
    });
}

EB_API eagle_backend_status eagle_backend_launcher_graph_destroy(uint64_t graph)
{
    return guarded([&] {
        if (graph != 0)
            cudaCheck(cudaGraphDestroy(reinterpret_cast<cudaGraph_t>(graph)), "cudaGraphDestroy");
    });
}

EB_API void eagle_backend_launcher_release(eagle_backend_launcher h)
{
    auto* l = reinterpret_cast<Launcher*>(h);
    if (l == nullptr || l->tag != kLauncher)
        return;
    int prev = -1;
    if (cudaGetDevice(&prev) == cudaSuccess)
        (void)cudaSetDevice(l->device);
    if (l->exec != nullptr)
        (void)cudaGraphExecDestroy(l->exec);
    (void)cudaGetLastError();
    if (prev >= 0)
        (void)cudaSetDevice(prev);
    retire(l);
}
