/*
 * ov_runtime.h - C-ABI device runtime of omnivoice-b200.
 *
 * Replaces the HIP helper layer of the reference generator
 * (device.hpp:16-77): `GpuError`/`Check` become integer status codes plus a
 * thread-local message, and `DeviceBuffer<T>` is rebuilt in C++ on top of
 * ov_malloc / ov_free (omnivoice_b200/csrc/host/device.hpp).  Every function
 * returns OV_OK (0) on success and never throws across the ABI.  Streams are
 * plain cudaStream_t values passed as opaque pointers, so a caller may hand in
 * a stream it created elsewhere (for example torch's current stream).
 */
#ifndef OMNIVOICE_B200_OV_RUNTIME_H_
#define OMNIVOICE_B200_OV_RUNTIME_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes shared by every entry point of the library. */
enum {
  OV_OK = 0,
  OV_ERR_INVALID = 1,     /* a size, pointer or shape check failed */
  OV_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  OV_ERR_OOM = 3,         /* device allocation failed */
  OV_ERR_UNSUPPORTED = 4, /* the model configuration is not implemented */
  OV_ERR_TIMEOUT = 5,     /* a bounded device-side wait ran out */
  OV_ERR_CANCELLED = 6,   /* the caller's cancellation callback fired */
  OV_ERR_IO = 7           /* a weight file could not be read */
};

typedef void* ov_stream_t; /* a cudaStream_t; NULL is the legacy stream */
typedef void* ov_event_t;  /* a cudaEvent_t */
typedef void* ov_graph_t;  /* an instantiated cudaGraphExec_t */

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to `capacity`) and returns the last status code.  Mirrors the
 * `what()` text of the reference's GpuError (device.hpp:16-30). */
int ov_last_error(char* buffer, size_t capacity);

int ov_device_count(int* count);
int ov_set_device(int device);
int ov_get_device(int* device);
/* Number of streaming multiprocessors and compute capability of `device`. */
int ov_device_info(int device, int* sm_count, int* major, int* minor);

/* device.hpp:43-58 (hipMalloc / hipFree of DeviceBuffer<T>). */
int ov_malloc(void** pointer, size_t bytes);
int ov_free(void* pointer);
int ov_malloc_host(void** pointer, size_t bytes); /* pinned */
int ov_free_host(void* pointer);

int ov_memcpy_h2d_async(void* dst, const void* src, size_t bytes, ov_stream_t stream);
int ov_memcpy_d2h_async(void* dst, const void* src, size_t bytes, ov_stream_t stream);
int ov_memcpy_d2d_async(void* dst, const void* src, size_t bytes, ov_stream_t stream);
int ov_memset_async(void* dst, int value, size_t bytes, ov_stream_t stream);

/* generator.cpp:385 creates one non-blocking stream per Generator. */
int ov_stream_create(ov_stream_t* stream);
int ov_stream_destroy(ov_stream_t stream);
int ov_stream_sync(ov_stream_t stream);

int ov_event_create(ov_event_t* event);
int ov_event_destroy(ov_event_t event);
int ov_event_record(ov_event_t event, ov_stream_t stream);
int ov_event_sync(ov_event_t event);
int ov_event_elapsed_ms(ov_event_t begin, ov_event_t end, float* milliseconds);

/* CUDA graphs (no counterpart in the reference, which launches every
 * kernel each step): ov_graph_capture_begin starts a thread-local capture
 * of `stream` (which must not be the legacy stream); ov_graph_capture_end
 * ends it and instantiates the captured work as *graph; ov_graph_launch
 * replays it on `stream`. */
int ov_graph_capture_begin(ov_stream_t stream);
int ov_graph_capture_end(ov_stream_t stream, ov_graph_t* graph);
int ov_graph_launch(ov_graph_t graph, ov_stream_t stream);
int ov_graph_destroy(ov_graph_t graph);

/* Bits of the device-side error word. */
enum {
  OV_DEVICE_WAIT_TIMEOUT = 1, /* a bounded wait ran out (no kernel of this library traps) */
  OV_DEVICE_BAD_ARGUMENT = 2  /* an index outside its range was skipped (a RoPE position,
                                 an attention work item's sequence) */
};

/* Device-side error word written by kernels (bits above).  Reads and
 * clears it on the current device's context; `*flags` is 0 when nothing
 * was reported. */
int ov_take_device_errors(uint32_t* flags, ov_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OMNIVOICE_B200_OV_RUNTIME_H_ */
