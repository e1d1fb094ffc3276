// CUDA runtime wrappers of the b2 C-ABI: device arena allocations, pinned
// staging, streams, events and graph capture.  The host C runtime never
// includes CUDA headers; it calls these.
#include <stdarg.h>
#include <stdio.h>

#include "b2_common.cuh"

static thread_local char g_err[512];

int b2_set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int b2_check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return 0;
}

extern "C" {

const char* b2_last_error(void) { return g_err; }

int b2_device_count(int* n) {
    B2_TRY(cudaGetDeviceCount(n));
    return 0;
}

int b2_set_device(int dev) {
    B2_TRY(cudaSetDevice(dev));
    return 0;
}

int b2_get_device(int* dev) {
    B2_TRY(cudaGetDevice(dev));
    return 0;
}

int b2_sm_count(int* n) {
    int dev;
    B2_TRY(cudaGetDevice(&dev));
    B2_TRY(cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev));
    return 0;
}

int b2_malloc(void** ptr, size_t bytes) {
    *ptr = nullptr;
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return b2_set_error(-2, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    return 0;
}

int b2_free(void* ptr) {
    if (ptr) B2_TRY(cudaFree(ptr));
    return 0;
}

int b2_host_alloc(void** ptr, size_t bytes) {
    *ptr = nullptr;
    cudaError_t e = cudaMallocHost(ptr, bytes ? bytes : 64);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return b2_set_error(-2, "cudaMallocHost(%zu): %s", bytes, cudaGetErrorString(e));
    }
    return 0;
}

int b2_host_free(void* ptr) {
    if (ptr) B2_TRY(cudaFreeHost(ptr));
    return 0;
}

int b2_mem_get_info(size_t* free_bytes, size_t* total_bytes) {
    B2_TRY(cudaMemGetInfo(free_bytes, total_bytes));
    return 0;
}

int b2_memcpy_h2d(void* dst, const void* src, size_t bytes, b2_stream_t s) {
    B2_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)s));
    return 0;
}

int b2_memcpy_d2h(void* dst, const void* src, size_t bytes, b2_stream_t s) {
    B2_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)s));
    return 0;
}

int b2_memcpy_d2d(void* dst, const void* src, size_t bytes, b2_stream_t s) {
    B2_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)s));
    return 0;
}

int b2_memset(void* dst, int value, size_t bytes, b2_stream_t s) {
    B2_TRY(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)s));
    return 0;
}

int b2_stream_create(b2_stream_t* s) {
    cudaStream_t st;
    B2_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    *s = (b2_stream_t)st;
    return 0;
}

int b2_stream_destroy(b2_stream_t s) {
    if (s) B2_TRY(cudaStreamDestroy((cudaStream_t)s));
    return 0;
}

int b2_stream_sync(b2_stream_t s) {
    B2_TRY(cudaStreamSynchronize((cudaStream_t)s));
    return 0;
}

int b2_stream_query(b2_stream_t s) {
    const cudaError_t e = cudaStreamQuery((cudaStream_t)s);
    if (e == cudaSuccess) return 0;
    if (e == cudaErrorNotReady) return 1;
    return b2_set_error(B2_ERR_CUDA, "cudaStreamQuery: %s", cudaGetErrorString(e));
}

int b2_event_create(b2_event_t* e) {
    cudaEvent_t ev;
    B2_TRY(cudaEventCreate(&ev));
    *e = (b2_event_t)ev;
    return 0;
}

int b2_event_destroy(b2_event_t e) {
    if (e) B2_TRY(cudaEventDestroy((cudaEvent_t)e));
    return 0;
}

// Inside a capture the record becomes an event-record node of the graph, so
// elapsed times between two such events time graph segments on the device.
int b2_event_record(b2_event_t e, b2_stream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    B2_TRY(cudaStreamIsCapturing((cudaStream_t)s, &st));
    if (st == cudaStreamCaptureStatusActive)
        B2_TRY(cudaEventRecordWithFlags((cudaEvent_t)e, (cudaStream_t)s, cudaEventRecordExternal));
    else
        B2_TRY(cudaEventRecord((cudaEvent_t)e, (cudaStream_t)s));
    return 0;
}

int b2_event_elapsed_ms(float* ms, b2_event_t a, b2_event_t b) {
    B2_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)a, (cudaEvent_t)b));
    return 0;
}

int b2_graph_begin(b2_stream_t s) {
    B2_TRY(cudaStreamBeginCapture((cudaStream_t)s, cudaStreamCaptureModeThreadLocal));
    return 0;
}

int b2_graph_end(b2_stream_t s, b2_graph_t* g) {
    cudaGraph_t graph;
    B2_TRY(cudaStreamEndCapture((cudaStream_t)s, &graph));
    cudaGraphExec_t exec;
    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
    *g = (b2_graph_t)exec;
    return 0;
}

int b2_graph_launch(b2_graph_t g, b2_stream_t s) {
    B2_TRY(cudaGraphLaunch((cudaGraphExec_t)g, (cudaStream_t)s));
    return 0;
}

int b2_graph_destroy(b2_graph_t g) {
    if (g) B2_TRY(cudaGraphExecDestroy((cudaGraphExec_t)g));
    return 0;
}

}  // extern "C"
