/*
 * wginfer.h — the type vocabulary the wGInfer op surface is written in.
 *
 * The enumerators and their values are those of the reference's public header
 * (include/wginfer.h:23-61 in wGInfer) so that a pointer, a dtype code or a
 * stream handle passes unchanged between the reference's C++ tensor runtime
 * and this backend. Nothing here is B200-specific.
 */
#ifndef __WGINFER_H__
#define __WGINFER_H__

#if defined(_WIN32)
#define __export __declspec(dllexport)
#elif defined(__GNUC__) && ((__GNUC__ >= 4) || (__GNUC__ == 3 && __GNUC_MINOR__ >= 3))
#define __export __attribute__((visibility("default")))
#else
#define __export
#endif

#ifdef __cplusplus
#define __C extern "C"
#include <cstddef>
#include <cstdint>
#else
#define __C
#include <stddef.h>
#include <stdint.h>
#endif

typedef enum {
    WGINFER_DEVICE_CPU = 0,
    WGINFER_DEVICE_NVIDIA = 1,
    WGINFER_DEVICE_METAX = 2,
    WGINFER_DEVICE_TYPE_COUNT
} wginferDeviceType_t;

typedef enum {
    WGINFER_DTYPE_INVALID = 0,
    WGINFER_DTYPE_BYTE = 1,
    WGINFER_DTYPE_BOOL = 2,
    WGINFER_DTYPE_I8 = 3,
    WGINFER_DTYPE_I16 = 4,
    WGINFER_DTYPE_I32 = 5,
    WGINFER_DTYPE_I64 = 6,
    WGINFER_DTYPE_U8 = 7,
    WGINFER_DTYPE_U16 = 8,
    WGINFER_DTYPE_U32 = 9,
    WGINFER_DTYPE_U64 = 10,
    WGINFER_DTYPE_F8 = 11,
    WGINFER_DTYPE_F16 = 12,
    WGINFER_DTYPE_F32 = 13,
    WGINFER_DTYPE_F64 = 14,
    WGINFER_DTYPE_BF16 = 15,
} wginferDataType_t;

/* A stream handle; on the NVIDIA device it is a cudaStream_t (NULL = legacy
 * default stream). */
typedef void *wginferStream_t;

typedef enum {
    WGINFER_MEMCPY_H2H = 0,
    WGINFER_MEMCPY_H2D = 1,
    WGINFER_MEMCPY_D2H = 2,
    WGINFER_MEMCPY_D2D = 3,
} wginferMemcpyKind_t;

#endif /* __WGINFER_H__ */
