#ifndef QWN_CUDA_ABI_H
#define QWN_CUDA_ABI_H

/*
 * Versioned C ABI between qwnrun and qwn_cuda.so (ABI version 1).
 *
 * This is the boundary the reference decoder binds at run time: qwnrun
 * dlopen()s qwn_cuda.so from its own directory and resolves the 17
 * qwn_cuda_abi_* symbols below (reference c/qwanto_decode.c:267-462).  The
 * structure layouts, constants, status codes and capability bits must be
 * byte-identical to the reference contract c/cuda/qwn_cuda_abi.h:27-274, so
 * they are restated here unchanged in meaning; the implementation behind
 * them (qwanto_b200/csrc/abi_v1.cu) is this project's own.
 *
 * No CUDA runtime types appear here.  Every structure starts with
 * QwnCudaAbiHeader; callees accept struct_size >= the size they know.
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32) && defined(QWN_CUDA_BUILDING_DLL)
#define QWN_CUDA_ABI_API __declspec(dllexport)
#elif defined(__GNUC__)
#define QWN_CUDA_ABI_API __attribute__((visibility("default")))
#else
#define QWN_CUDA_ABI_API
#endif

#define QWN_CUDA_ABI_VERSION 1u
#define QWN_CUDA_ABI_NAME "qwn_cuda_hypervsq2"
#define QWN_CUDA_HYPERVSQ2_BLOCK_BYTES 74u
#define QWN_CUDA_HYPERVSQ2_BLOCK_ELEMENTS 256u
#define QWN_CUDA_MAX_RESIDENT_TENSORS 512u
#define QWN_CUDA_MAX_RESIDENT_KV_CACHES 128u

typedef struct {
    uint32_t struct_size;
    uint32_t abi_version;
    uint32_t reserved[4];
} QwnCudaAbiHeader;

static inline void qwn_cuda_abi_header_init(QwnCudaAbiHeader *header, uint32_t struct_size) {
    if (!header) return;
    header->struct_size = struct_size;
    header->abi_version = QWN_CUDA_ABI_VERSION;
    header->reserved[0] = header->reserved[1] = header->reserved[2] = header->reserved[3] = 0;
}

/* capability bits (reference c/cuda/qwn_cuda_abi.h:51-58); bits 6 and up
 * are this library's extensions, declared in qwn_kv_b200.h */
enum {
    QWN_CUDA_CAP_HYPERVSQ2_GEMV = 1ull << 0,
    QWN_CUDA_CAP_HYPERVSQ2_GEMM = 1ull << 1,
    QWN_CUDA_CAP_RESIDENT_WEIGHTS = 1ull << 2,
    QWN_CUDA_CAP_TELEMETRY = 1ull << 3,
    QWN_CUDA_CAP_DEVICE_ENUMERATION = 1ull << 4,
    QWN_CUDA_CAP_Q8_KV = 1ull << 5
};

typedef enum {
    QWN_CUDA_STATUS_OK = 0,
    QWN_CUDA_STATUS_INVALID_ARGUMENT = -1,
    QWN_CUDA_STATUS_ABI_MISMATCH = -2,
    QWN_CUDA_STATUS_UNAVAILABLE = -3,
    QWN_CUDA_STATUS_OUT_OF_MEMORY = -4,
    QWN_CUDA_STATUS_UNSUPPORTED = -5,
    QWN_CUDA_STATUS_RUNTIME_ERROR = -6
} QwnCudaStatus;

typedef enum { QWN_CUDA_TENSOR_HYPERVSQ2_74 = 1 } QwnCudaTensorDType;
typedef enum { QWN_CUDA_INPUT_Q8 = 1 } QwnCudaInputMode;

typedef struct {
    QwnCudaAbiHeader header;
    uint64_t capability_bits;
    uint32_t max_devices;
    uint32_t max_resident_tensors;
    uint32_t hypervsq2_block_bytes;
    uint32_t hypervsq2_block_elements;
    char abi_name[32];
} QwnCudaAbiInfo;

typedef struct {
    QwnCudaAbiHeader header;
    int32_t device_id;
    int32_t compute_major;
    int32_t compute_minor;
    uint64_t total_vram_bytes;
    uint64_t free_vram_bytes;
    char name[128];
    char driver[64];
} QwnCudaDeviceInfo;

typedef struct {
    QwnCudaAbiHeader header;
    int32_t device_id;
    uint32_t flags;
    uint64_t memory_budget_bytes;
    uint64_t context_size;
} QwnCudaContextOptions;

typedef struct { QwnCudaAbiHeader header; void *opaque; } QwnCudaContextHandle;
typedef struct { QwnCudaAbiHeader header; void *opaque; } QwnCudaTensorHandle;
typedef struct { QwnCudaAbiHeader header; void *opaque; } QwnCudaKvCacheHandle;

typedef struct {
    QwnCudaAbiHeader header;
    uint32_t max_tokens;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t reserved;
} QwnCudaKvCacheOptions;

typedef struct {
    QwnCudaAbiHeader header;
    QwnCudaKvCacheHandle cache;
    const float *host_key;
    const float *host_value;
    uint32_t n_channels;
    uint32_t token;
} QwnCudaKvAppendRequest;

typedef struct {
    QwnCudaAbiHeader header;
    QwnCudaKvCacheHandle cache;
    const float *host_query;
    float *host_output;
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t position;
    float scale;
} QwnCudaKvAttentionRequest;

typedef struct {
    QwnCudaAbiHeader header;
    const void *host_data;
    uint64_t data_bytes;
    uint32_t dtype;
    uint32_t rows;
    uint32_t cols;
    uint32_t block_bytes;
} QwnCudaTensorUpload;

typedef struct {
    QwnCudaAbiHeader header;
    QwnCudaTensorHandle tensor;
    const int8_t *input_q8;
    float input_scale;
    const float *input_scales;
    float *output;
    uint32_t batch;
    uint32_t rows;
    uint32_t cols;
    uint32_t input_stride;
    uint32_t output_stride;
    uint32_t input_mode;
} QwnCudaGemmRequest;

typedef struct {
    QwnCudaAbiHeader header;
    uint64_t gpu_matmul_count;
    uint64_t gpu_kernel_launch_count;
    uint64_t gpu_projection_count;
    uint64_t gpu_upload_count;
    uint64_t gpu_upload_bytes;
    uint64_t gpu_resident_bytes;
    uint64_t cpu_matmul_fallback_count;
    uint64_t unsupported_projection_count;
    double gpu_kernel_ms;
    double gpu_transfer_ms;
    double gpu_sync_ms;
    int32_t device_id;
    uint32_t reserved_device;
    char device_name[128];
    char kernel_type[32];
    char dll_hash[65];
    uint64_t kv_cache_kernel_count;
    uint64_t kv_cache_upload_bytes;
    uint64_t kv_cache_resident_bytes;
    double kv_cache_kernel_ms;
    double kv_cache_transfer_ms;
    char kv_cache_kernel_type[32];
} QwnCudaTelemetry;

typedef int (*QwnCudaAbiQueryFn)(QwnCudaAbiInfo *info);
typedef int (*QwnCudaCapabilityQueryFn)(QwnCudaAbiInfo *info);
typedef int (*QwnCudaEnumerateDevicesFn)(QwnCudaDeviceInfo *devices, uint32_t capacity,
                                         uint32_t *count);
typedef int (*QwnCudaContextCreateFn)(const QwnCudaContextOptions *options,
                                      QwnCudaContextHandle *context);
typedef int (*QwnCudaContextDestroyFn)(QwnCudaContextHandle *context);
typedef int (*QwnCudaTensorUploadFn)(QwnCudaContextHandle *context,
                                     const QwnCudaTensorUpload *upload,
                                     QwnCudaTensorHandle *tensor);
typedef int (*QwnCudaTensorReleaseFn)(QwnCudaContextHandle *context, QwnCudaTensorHandle *tensor);
typedef int (*QwnCudaKvCreateFn)(QwnCudaContextHandle *context, const QwnCudaKvCacheOptions *options,
                                 QwnCudaKvCacheHandle *cache);
typedef int (*QwnCudaKvDestroyFn)(QwnCudaContextHandle *context, QwnCudaKvCacheHandle *cache);
typedef int (*QwnCudaKvAppendFn)(QwnCudaContextHandle *context, const QwnCudaKvAppendRequest *request,
                                 QwnCudaTelemetry *telemetry);
typedef int (*QwnCudaKvAttentionFn)(QwnCudaContextHandle *context,
                                    const QwnCudaKvAttentionRequest *request,
                                    QwnCudaTelemetry *telemetry);
typedef int (*QwnCudaKvResetFn)(QwnCudaContextHandle *context, QwnCudaKvCacheHandle *cache);
typedef int (*QwnCudaGemvFn)(QwnCudaContextHandle *context, const QwnCudaGemmRequest *request,
                             QwnCudaTelemetry *telemetry);
typedef int (*QwnCudaGemmFn)(QwnCudaContextHandle *context, const QwnCudaGemmRequest *request,
                             QwnCudaTelemetry *telemetry);
typedef int (*QwnCudaSynchronizeFn)(QwnCudaContextHandle *context);
typedef int (*QwnCudaTelemetryFn)(QwnCudaContextHandle *context, QwnCudaTelemetry *telemetry);
typedef int (*QwnCudaLastErrorFn)(char *buffer, uint32_t buffer_size);

/* Each entry point replaces the same-named reference export of
 * c/cuda/qwn_hypervsq2_cuda_abi.cu (line of the reference definition). */
QWN_CUDA_ABI_API int qwn_cuda_abi_query(QwnCudaAbiInfo *info);                      /* :417 */
QWN_CUDA_ABI_API int qwn_cuda_abi_get_capabilities(QwnCudaAbiInfo *info);           /* :438 */
QWN_CUDA_ABI_API int qwn_cuda_abi_enumerate_devices(QwnCudaDeviceInfo *devices,
                                                     uint32_t capacity, uint32_t *count); /* :442 */
QWN_CUDA_ABI_API int qwn_cuda_abi_context_create(const QwnCudaContextOptions *options,
                                                  QwnCudaContextHandle *context);    /* :477 */
QWN_CUDA_ABI_API int qwn_cuda_abi_context_destroy(QwnCudaContextHandle *context);   /* :504 */
QWN_CUDA_ABI_API int qwn_cuda_abi_upload_tensor(QwnCudaContextHandle *context,
                                                 const QwnCudaTensorUpload *upload,
                                                 QwnCudaTensorHandle *tensor);       /* :537 */
QWN_CUDA_ABI_API int qwn_cuda_abi_release_tensor(QwnCudaContextHandle *context,
                                                  QwnCudaTensorHandle *tensor);      /* :587 */
QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_create(QwnCudaContextHandle *context,
                                                   const QwnCudaKvCacheOptions *options,
                                                   QwnCudaKvCacheHandle *cache);     /* :604 */
QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_destroy(QwnCudaContextHandle *context,
                                                    QwnCudaKvCacheHandle *cache);    /* :812 */
QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_append(QwnCudaContextHandle *context,
                                                   const QwnCudaKvAppendRequest *request,
                                                   QwnCudaTelemetry *telemetry);     /* :692 */
QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_attention(QwnCudaContextHandle *context,
                                                      const QwnCudaKvAttentionRequest *request,
                                                      QwnCudaTelemetry *telemetry);  /* :749 */
QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_reset(QwnCudaContextHandle *context,
                                                  QwnCudaKvCacheHandle *cache);      /* :803 */
QWN_CUDA_ABI_API int qwn_cuda_abi_hypervsq2_gemv(QwnCudaContextHandle *context,
                                                  const QwnCudaGemmRequest *request,
                                                  QwnCudaTelemetry *telemetry);      /* :835 */
QWN_CUDA_ABI_API int qwn_cuda_abi_hypervsq2_gemm(QwnCudaContextHandle *context,
                                                  const QwnCudaGemmRequest *request,
                                                  QwnCudaTelemetry *telemetry);      /* :845 */
QWN_CUDA_ABI_API int qwn_cuda_abi_synchronize(QwnCudaContextHandle *context);       /* :854 */
QWN_CUDA_ABI_API int qwn_cuda_abi_get_telemetry(QwnCudaContextHandle *context,
                                                 QwnCudaTelemetry *telemetry);       /* :865 */
QWN_CUDA_ABI_API int qwn_cuda_abi_last_error(char *buffer, uint32_t buffer_size);   /* :874 */

#ifdef __cplusplus
}
#endif

#endif /* QWN_CUDA_ABI_H */
