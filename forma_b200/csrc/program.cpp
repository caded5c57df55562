// Prepared programs: a sequence of fb_* calls recorded once on a stream and
// replayed as one CUDA graph launch.
//
// The reference prepares typed programs and optionally captures them into a
// CUDA graph that is replayed with the same buffers (compute-cuda/src/
// program.rs:1-60, program/graph.rs, program/execution.rs:20-150): steps are
// validated and their scratch reserved at preparation, replay allocates
// nothing, and an execution error poisons the program for good.  Here any
// sequence of this library's entry points - convolution included, which the
// reference's program builder lacks - is recorded by stream capture.  Every
// entry point is capture-safe: library scratch is never allocated while its
// stream is capturing (the call fails instead), so one eager call with the
// same shapes on the same stream must come first.
#include <cuda_runtime.h>

#include <string>

#include "host.h"
#include "kernels.h"

struct fb_program {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;  // this library's kernels in the recording
    uint64_t nodes = 0;     // graph nodes (kernels, memsets, other libraries' work)
    int device = -1;
    bool poisoned = false;
};

namespace fb {
namespace {

thread_local void* g_capture_stream = nullptr;
thread_local bool g_capturing = false;
thread_local uint64_t g_capture_launches0 = 0;

int cuda_fail(cudaError_t e, int status, const char* what) {
    return fail(status, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int fb_program_begin(void* stream) {
    if (!stream || stream == static_cast<void*>(cudaStreamPerThread))
        return fail(FB_ERR_INVALID_INPUT, "a program records on a created stream, not a default stream");
    if (g_capturing) return fail(FB_ERR_INVALID_INPUT, "this thread is already recording a program");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaError_t e = cudaStreamIsCapturing(s, &cap); e != cudaSuccess)
        return cuda_fail(e, FB_ERR_DRIVER, "cudaStreamIsCapturing");
    if (cap != cudaStreamCaptureStatusNone) return fail(FB_ERR_INVALID_INPUT, "the stream is already capturing");
    // Thread-local mode: other threads' unsafe calls do not break this
    // recording, and this thread may not make such calls (cudaMalloc among
    // them) while recording.
    if (cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal); e != cudaSuccess)
        return cuda_fail(e, FB_ERR_GRAPH, "cudaStreamBeginCapture");
    g_capture_stream = stream;
    g_capturing = true;
    g_capture_launches0 = thread_launch_count();
    return FB_OK;
}

int fb_program_end(void* stream, fb_program** program) {
    if (!g_capturing || stream != g_capture_stream)
        return fail(FB_ERR_INVALID_INPUT, "no program is being recorded on this stream by this thread");
    g_capturing = false;
    g_capture_stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph);
    if (e != cudaSuccess || !graph) {
        (void)cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        return cuda_fail(e == cudaSuccess ? cudaErrorStreamCaptureInvalidated : e, FB_ERR_GRAPH,
                         "recording invalidated (an allocation or a synchronising call while recording?)");
    }
    if (!program) {
        cudaGraphDestroy(graph);
        return fail(FB_ERR_INVALID_INPUT, "null program pointer");
    }
    fb_program* p = new fb_program;
    p->graph = graph;
    p->launches = thread_launch_count() - g_capture_launches0;
    size_t n = 0;
    cudaGraphGetNodes(graph, nullptr, &n);
    p->nodes = n;
    cudaGetDevice(&p->device);
    if (cudaError_t ie = cudaGraphInstantiate(&p->exec, graph, 0); ie != cudaSuccess) {
        (void)cudaGetLastError();
        cudaGraphDestroy(graph);
        delete p;
        return cuda_fail(ie, FB_ERR_GRAPH, "cudaGraphInstantiate");
    }
    *program = p;
    return FB_OK;
}

int fb_program_launch(fb_program* program, void* stream) {
    begin_route();
    if (!program) return fail(FB_ERR_INVALID_INPUT, "null program");
    if (program->poisoned)
        return fail(FB_ERR_PROGRAM_POISONED, "prepared program is poisoned after an execution error");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != program->device)
        return fail(FB_ERR_FOREIGN_RUNTIME, "the program was recorded on device " + std::to_string(program->device) +
                                                ", the call runs on device " + std::to_string(dev));
    if (cudaError_t e = cudaGraphLaunch(program->exec, static_cast<cudaStream_t>(stream)); e != cudaSuccess) {
        program->poisoned = true;
        return cuda_fail(e, FB_ERR_DRIVER, "cudaGraphLaunch");
    }
    return FB_OK;
}

int fb_program_stats(const fb_program* program, uint64_t* kernel_launches, uint64_t* graph_nodes, int32_t* poisoned) {
    if (!program) return fail(FB_ERR_INVALID_INPUT, "null program");
    if (kernel_launches) *kernel_launches = program->launches;
    if (graph_nodes) *graph_nodes = program->nodes;
    if (poisoned) *poisoned = program->poisoned ? 1 : 0;
    return FB_OK;
}

int fb_program_destroy(fb_program* program) {
    if (!program) return FB_OK;
    int rc = FB_OK;
    if (program->exec && cudaGraphExecDestroy(program->exec) != cudaSuccess) rc = FB_ERR_DRIVER;
    if (program->graph && cudaGraphDestroy(program->graph) != cudaSuccess) rc = FB_ERR_DRIVER;
    delete program;
    return rc == FB_OK ? FB_OK : fail(rc, "graph destruction failed");
}

}  // extern "C"
