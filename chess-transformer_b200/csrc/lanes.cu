// The batch runtime of include/fry_b200.h's fry_lanes_*: `Lane` and `GraphedBatches` (engine/inference.py:85-225) in
// C++, with the CUDA runtime calls engine/cuda_runtime.py makes for the Rust round loop (cudaMemcpyAsync, cudaGraphLaunch,
// cudaEventRecord, cudaEventSynchronize, cudaStreamSynchronize). Each lane records fry_forward (or fry_forward_lean) once
// per batch size into a CUDA graph on its own stream. Every size's graph reads the lane's one rows buffer and writes its
// one answers buffer, and shares its one workspace, which is safe because a lane has at most one batch out.
#include <algorithm>
#include <cstring>
#include <vector>

namespace {

struct Lane {
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    void* rows_host = nullptr;
    float* answers_host = nullptr;
    void* rows = nullptr;
    float* answers = nullptr;
    void* workspace = nullptr;
    std::vector<cudaGraphExec_t> graphs;  // one per size
    bool pending = false;
    int count = 0;
};

}  // namespace

struct FryLanes {
    int device = 0;
    bool lean = false, blocking_wait = false;
    size_t row_bytes = 0, answer_bytes = 0;
    std::vector<int> sizes;
    std::vector<Lane> lanes;
};

namespace {

void release(FryLanes* lanes) {
    cudaSetDevice(lanes->device);
    for (Lane& lane : lanes->lanes) {
        if (lane.stream) cudaStreamSynchronize(lane.stream);
        for (cudaGraphExec_t graph : lane.graphs)
            if (graph) cudaGraphExecDestroy(graph);
        if (lane.done) cudaEventDestroy(lane.done);
        if (lane.stream) cudaStreamDestroy(lane.stream);
        cudaFreeHost(lane.rows_host);
        cudaFreeHost(lane.answers_host);
        cudaFree(lane.rows);
        cudaFree(lane.answers);
        cudaFree(lane.workspace);
    }
    delete lanes;
}

// The lane's forward for `size` boards on its stream: what each graph records.
int lane_forward(const FryNetwork* network, const FryLanes* lanes, const Lane& lane, int size, size_t workspace_bytes) {
    return lanes->lean ? fry_forward_lean(network, static_cast<const uint8_t*>(lane.rows), size, lane.answers, lane.workspace,
                                          workspace_bytes, lane.stream)
                       : fry_forward(network, static_cast<const int64_t*>(lane.rows), size, lane.answers, lane.workspace,
                                     workspace_bytes, lane.stream);
}

// Allocates a lane's buffers and records its graphs. The rows start zeroed: token 0 and answer column 0 are in range, so
// the warm-up runs on valid boards.
int build_lane(const FryNetwork* network, FryLanes* lanes, Lane& lane, bool warm_up) {
    const int largest = lanes->sizes.back();
    const size_t workspace_bytes =
        lanes->lean ? fry_forward_lean_workspace_bytes(network, largest) : fry_forward_workspace_bytes(network, largest);
    int status;
    if ((status = check(cudaStreamCreateWithFlags(&lane.stream, cudaStreamNonBlocking), "fry_lanes_create: a lane's stream")) ||
        (status = check(cudaEventCreateWithFlags(&lane.done, cudaEventDisableTiming | (lanes->blocking_wait ? cudaEventBlockingSync : 0)),
                        "fry_lanes_create: a lane's event")) ||
        (status = check(cudaHostAlloc(&lane.rows_host, largest * lanes->row_bytes, cudaHostAllocDefault), "fry_lanes_create: pinned rows")) ||
        (status = check(cudaHostAlloc(reinterpret_cast<void**>(&lane.answers_host), largest * lanes->answer_bytes, cudaHostAllocDefault),
                        "fry_lanes_create: pinned answers")) ||
        (status = check(cudaMalloc(&lane.rows, largest * lanes->row_bytes), "fry_lanes_create: device rows")) ||
        (status = check(cudaMalloc(reinterpret_cast<void**>(&lane.answers), largest * lanes->answer_bytes), "fry_lanes_create: device answers")) ||
        (status = check(cudaMalloc(&lane.workspace, workspace_bytes), "fry_lanes_create: the workspace")))
        return status;
    std::memset(lane.rows_host, 0, largest * lanes->row_bytes);
    if ((status = check(cudaMemsetAsync(lane.rows, 0, largest * lanes->row_bytes, lane.stream), "fry_lanes_create: zeroing the rows")))
        return status;
    // the first lane's warm-up sets every kernel's attributes before any capture (engine/inference.py:111-115)
    if (warm_up)
        for (int size : lanes->sizes)
            if ((status = lane_forward(network, lanes, lane, size, workspace_bytes))) return status;
    if ((status = check(cudaStreamSynchronize(lane.stream), "fry_lanes_create: the warm-up"))) return status;
    lane.graphs.assign(lanes->sizes.size(), nullptr);
    for (size_t i = lanes->sizes.size(); i-- > 0;) {
        cudaGraph_t graph = nullptr;
        if ((status = check(cudaStreamBeginCapture(lane.stream, cudaStreamCaptureModeThreadLocal), "fry_lanes_create: a capture")))
            return status;
        const int recorded = lane_forward(network, lanes, lane, lanes->sizes[i], workspace_bytes);
        const std::string recorded_error = recorded ? g_last_error : std::string();
        const cudaError_t ended = cudaStreamEndCapture(lane.stream, &graph);
        if (recorded) {
            if (graph) cudaGraphDestroy(graph);
            return fail(recorded, "fry_lanes_create: recording size " + std::to_string(lanes->sizes[i]) + ": " + recorded_error);
        }
        if ((status = check(ended, "fry_lanes_create: ending a capture"))) return status;
        status = check(cudaGraphInstantiate(&lane.graphs[i], graph, 0), "fry_lanes_create: instantiating a graph");
        cudaGraphDestroy(graph);
        if (status) return status;
    }
    return check(cudaEventRecord(lane.done, lane.stream), "fry_lanes_create: the first record");
}

Lane* lane_at(const FryLanes* lanes, int lane, const char* what) {
    if (!lanes || lane < 0 || lane >= static_cast<int>(lanes->lanes.size())) {
        fail(FRY_ERROR_SHAPE, std::string(what) + ": no such lane");
        return nullptr;
    }
    return const_cast<Lane*>(&lanes->lanes[lane]);
}

}  // namespace

extern "C" {

int fry_lanes_create(const FryNetwork* network, const int* sizes, int sizes_count, int in_flight, int lean, int blocking_wait,
                     FryLanes** lanes_out) {
    if (!network || !sizes || sizes_count <= 0 || in_flight <= 0 || !lanes_out)
        return fail(FRY_ERROR_SHAPE, "fry_lanes_create needs a network, at least one size and one lane");
    for (int i = 0; i < sizes_count; ++i)
        if (sizes[i] <= 0 || (i > 0 && sizes[i] <= sizes[i - 1]))
            return fail(FRY_ERROR_SHAPE, "fry_lanes_create takes positive sizes in ascending order");
    *lanes_out = nullptr;
    FryLanes* lanes = new FryLanes;
    lanes->lean = lean != 0;
    lanes->blocking_wait = blocking_wait != 0;
    lanes->row_bytes = lanes->lean ? fry::kLeanRow : 70 * sizeof(int64_t);
    lanes->answer_bytes = (lanes->lean ? fry::kLeanColumns : kAnswerWidth) * sizeof(float);
    lanes->sizes.assign(sizes, sizes + sizes_count);
    int status = check(cudaGetDevice(&lanes->device), "fry_lanes_create: the current device");
    lanes->lanes.resize(status ? 0 : in_flight);
    for (int i = 0; !status && i < in_flight; ++i) status = build_lane(network, lanes, lanes->lanes[i], i == 0);
    if (status) {
        const std::string message = g_last_error;
        release(lanes);
        return fail(status, message);
    }
    *lanes_out = lanes;
    g_last_error.clear();
    return FRY_OK;
}

int fry_lanes_destroy(FryLanes* lanes) {
    if (lanes) release(lanes);
    g_last_error.clear();
    return FRY_OK;
}

int fry_lanes_free_lane(const FryLanes* lanes, int* lane) {
    if (!lanes || !lane) return fail(FRY_ERROR_SHAPE, "fry_lanes_free_lane needs lanes and an out pointer");
    for (size_t i = 0; i < lanes->lanes.size(); ++i)
        if (!lanes->lanes[i].pending) {
            *lane = static_cast<int>(i);
            g_last_error.clear();
            return FRY_OK;
        }
    return fail(FRY_ERROR_STATE, "more batches in flight than lanes");
}

int fry_lanes_handles(const FryLanes* lanes, int lane, FryLaneHandles* handles) {
    const Lane* l = lane_at(lanes, lane, "fry_lanes_handles");
    if (!l) return FRY_ERROR_SHAPE;
    if (!handles) return fail(FRY_ERROR_SHAPE, "fry_lanes_handles needs an out pointer");
    *handles = FryLaneHandles{lanes->device, l->stream, l->done, l->rows_host, l->rows, l->answers_host, l->answers};
    g_last_error.clear();
    return FRY_OK;
}

int fry_lanes_graph(const FryLanes* lanes, int lane, int size_index, void** graph_exec) {
    const Lane* l = lane_at(lanes, lane, "fry_lanes_graph");
    if (!l) return FRY_ERROR_SHAPE;
    if (!graph_exec || size_index < 0 || size_index >= static_cast<int>(l->graphs.size()))
        return fail(FRY_ERROR_SHAPE, "fry_lanes_graph: no such size");
    *graph_exec = l->graphs[size_index];
    g_last_error.clear();
    return FRY_OK;
}

int fry_lanes_launch(FryLanes* lanes, int lane, int count, int* size) {
    Lane* l = lane_at(lanes, lane, "fry_lanes_launch");
    if (!l) return FRY_ERROR_SHAPE;
    if (count <= 0 || count > lanes->sizes.back())
        return fail(FRY_ERROR_SHAPE, "fry_lanes_launch takes 1 to " + std::to_string(lanes->sizes.back()) + " boards, got " +
                                         std::to_string(count));
    if (l->pending) return fail(FRY_ERROR_STATE, "fry_lanes_launch: the lane's batch is still out");
    const size_t index = std::lower_bound(lanes->sizes.begin(), lanes->sizes.end(), count) - lanes->sizes.begin();
    int status;
    if ((status = check(cudaSetDevice(lanes->device), "the lane's device")) ||
        (status = check(cudaMemcpyAsync(l->rows, l->rows_host, count * lanes->row_bytes, cudaMemcpyHostToDevice, l->stream),
                        "the boards' copy")))
        return status;
    l->pending = true;
    l->count = count;
    if ((status = check(cudaGraphLaunch(l->graphs[index], l->stream), "the graph's launch")) ||
        (status = check(cudaEventRecord(l->done, l->stream), "the batch's event")))
        return status;
    if (size) *size = lanes->sizes[index];
    return FRY_OK;
}

int fry_lanes_collect(FryLanes* lanes, int lane, int* count) {
    Lane* l = lane_at(lanes, lane, "fry_lanes_collect");
    if (!l) return FRY_ERROR_SHAPE;
    if (!l->pending) return fail(FRY_ERROR_STATE, "fry_lanes_collect: the lane has no batch out");
    int status;
    if ((status = check(cudaSetDevice(lanes->device), "the lane's device"))) return status;
    if (lanes->blocking_wait && (status = check(cudaEventSynchronize(l->done), "the batch"))) return status;
    if ((status = check(cudaMemcpyAsync(l->answers_host, l->answers, l->count * lanes->answer_bytes, cudaMemcpyDeviceToHost, l->stream),
                        "the answers' copy")) ||
        (status = check(cudaStreamSynchronize(l->stream), "the batch")))
        return status;
    l->pending = false;
    if (count) *count = l->count;
    return FRY_OK;
}

int fry_lanes_settle(FryLanes* lanes) {
    if (!lanes) return fail(FRY_ERROR_SHAPE, "fry_lanes_settle needs lanes");
    int status;
    if ((status = check(cudaSetDevice(lanes->device), "the lanes' device"))) return status;
    for (Lane& lane : lanes->lanes)
        if (lane.pending) {
            if ((status = check(cudaStreamSynchronize(lane.stream), "a lane's batch"))) return status;
            lane.pending = false;
        }
    return FRY_OK;
}

}  // extern "C"
