/*
 * K1 kernel ABI v1 types, layout-identical to eshkol-transformer's
 * include/eshkol_transformer/kernel_abi.h (struct layouts frozen by the static
 * asserts at kernel_abi.h:176-234).  The layouts, field names, enum values and
 * limits must match the reference exactly: a K1 runtime built from the
 * reference (native/kernel_abi.c) discovers and dispatches the providers this
 * library exports through these very structs.  When the reference header is
 * included first, its definitions are used and this file only re-checks them.
 */
#ifndef ESHKOL_B200_KERNEL_ABI_V1_H
#define ESHKOL_B200_KERNEL_ABI_V1_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef ESHKOL_TRANSFORMER_KERNEL_ABI_H
#define ESHKOL_TRANSFORMER_KERNEL_ABI_H

#define ET_KERNEL_ABI_MAJOR 1u
#define ET_KERNEL_ABI_MINOR 0u
#define ET_KERNEL_PROVIDER_SYMBOL_V1 "eshkol_transformer_kernel_provider_v1"
#define ET_KERNEL_PROVIDER_KNOWN_REQUIRED_FEATURES UINT64_C(0)
#define ET_KERNEL_ERROR_OPERATION_CAPACITY 64u
#define ET_KERNEL_ERROR_MESSAGE_CAPACITY 192u
#define ET_KERNEL_MAX_CAPABILITIES 4096u
#define ET_KERNEL_MAX_LIST_ENTRIES 4096u
#define ET_KERNEL_MAX_SHAPE_RANGES 4096u
#define ET_KERNEL_MAX_RANK 64u
#define ET_KERNEL_MAX_TENSORS 1024u
#define ET_KERNEL_MAX_SYMBOL_BYTES 127u
#define ET_KERNEL_MAX_METADATA_BYTES 1024u
#define ET_KERNEL_CAPABILITY_V1_0_SIZE ((size_t)120u)
#define ET_KERNEL_TENSOR_VIEW_V1_0_SIZE ((size_t)72u)
#define ET_KERNEL_REQUEST_V1_0_SIZE ((size_t)56u)
#define ET_KERNEL_CALL_V1_0_SIZE ((size_t)88u)
#define ET_KERNEL_PROVIDER_V1_0_SIZE ((size_t)96u)

/* capability status */
enum {
  ET_KERNEL_CAPABILITY_UNVERIFIED = 0,
  ET_KERNEL_CAPABILITY_VERIFIED = 1,
  ET_KERNEL_CAPABILITY_UNSUPPORTED = 2
};
typedef uint32_t et_kernel_capability_status;

/* error categories (validate_call returns the category as int32) */
enum {
  ET_KERNEL_ERROR_NONE = 0,
  ET_KERNEL_ERROR_INVALID_ARGUMENT,
  ET_KERNEL_ERROR_SHAPE_MISMATCH,
  ET_KERNEL_ERROR_DTYPE_MISMATCH,
  ET_KERNEL_ERROR_DEVICE_MISMATCH,
  ET_KERNEL_ERROR_NONCONTIGUOUS,
  ET_KERNEL_ERROR_UNSUPPORTED,
  ET_KERNEL_ERROR_VERSION_MISMATCH,
  ET_KERNEL_ERROR_INTERNAL
};
typedef uint32_t et_kernel_error_category;

/* error codes */
enum {
  ET_KERNEL_CODE_OK = 0,
  ET_KERNEL_CODE_NULL_ARGUMENT,
  ET_KERNEL_CODE_INVALID_STRUCT_SIZE,
  ET_KERNEL_CODE_INVALID_TEXT,
  ET_KERNEL_CODE_INVALID_ENUM,
  ET_KERNEL_CODE_DUPLICATE_ENTRY,
  ET_KERNEL_CODE_SYMBOL_MISSING,
  ET_KERNEL_CODE_ABI_MAJOR_MISMATCH,
  ET_KERNEL_CODE_UNKNOWN_REQUIRED_FEATURE,
  ET_KERNEL_CODE_ALLOCATION_FAILED,
  ET_KERNEL_CODE_BUFFER_TOO_SMALL,
  ET_KERNEL_CODE_INTEGER_OVERFLOW,
  ET_KERNEL_CODE_INVALID_SHAPE,
  ET_KERNEL_CODE_INVALID_BUFFER,
  ET_KERNEL_CODE_ALIASING_OUTPUT,
  ET_KERNEL_CODE_CAPABILITY_NOT_VERIFIED,
  ET_KERNEL_CODE_PROVIDER_REJECTED
};
typedef uint32_t et_kernel_error_code;

typedef struct et_kernel_error {
  et_kernel_error_category category;
  et_kernel_error_code code;
  char operation[ET_KERNEL_ERROR_OPERATION_CAPACITY];
  char message[ET_KERNEL_ERROR_MESSAGE_CAPACITY];
} et_kernel_error;

typedef struct et_kernel_dimension_range_v1 {
  uint64_t minimum;
  uint64_t maximum;
  uint8_t maximum_unbounded;
  uint8_t reserved[7];
} et_kernel_dimension_range_v1;

typedef struct et_kernel_shape_range_v1 {
  size_t rank;
  const et_kernel_dimension_range_v1 *dimensions;
} et_kernel_shape_range_v1;

typedef struct et_kernel_capability_v1 {
  size_t struct_size;
  const char *name;
  et_kernel_capability_status status;
  const char *implementation;
  const char *version;
  const char *evidence;
  uint8_t deterministic;
  uint8_t reserved[7];
  size_t operation_count;
  const char *const *operations;
  size_t dtype_count;
  const char *const *dtypes;
  size_t device_count;
  const char *const *devices;
  size_t shape_range_count;
  const et_kernel_shape_range_v1 *shape_ranges;
} et_kernel_capability_v1;

enum { ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR = 1 };
typedef uint32_t et_kernel_layout_v1;

typedef struct et_kernel_tensor_view_v1 {
  size_t struct_size;
  void *data;
  size_t byte_length;
  const char *dtype;
  const char *device;
  et_kernel_layout_v1 layout;
  uint64_t offset_bytes;
  size_t rank;
  const uint64_t *shape;
} et_kernel_tensor_view_v1;

typedef struct et_kernel_request_v1 {
  size_t struct_size;
  const char *operation;
  const char *dtype;
  const char *device;
  size_t rank;
  const uint64_t *shape;
  uint8_t deterministic;
  uint8_t reserved[7];
} et_kernel_request_v1;

typedef struct et_kernel_call_v1 {
  size_t struct_size;
  const char *capability;
  const et_kernel_request_v1 *request;
  size_t input_count;
  size_t input_stride;
  size_t input_bytes;
  const void *inputs;
  size_t output_count;
  size_t output_stride;
  size_t output_bytes;
  void *outputs;
} et_kernel_call_v1;

typedef int32_t (*et_kernel_validate_call_v1)(const et_kernel_call_v1 *call,
                                              et_kernel_error *error);
typedef void (*et_kernel_invoke_call_v1)(const et_kernel_call_v1 *call);

typedef struct et_kernel_provider_v1 {
  size_t struct_size;
  uint32_t abi_major;
  uint32_t abi_minor;
  uint64_t required_features;
  const char *name;
  const char *version;
  const char *evidence;
  size_t capability_count;
  size_t capability_stride;
  size_t capability_bytes;
  const void *capabilities;
  et_kernel_validate_call_v1 validate_call;
  et_kernel_invoke_call_v1 invoke_call;
} et_kernel_provider_v1;

#endif /* ESHKOL_TRANSFORMER_KERNEL_ABI_H */

#if defined(__cplusplus)
#define ET_B200_ABI_ASSERT(c, m) static_assert(c, m)
#else
#define ET_B200_ABI_ASSERT(c, m) _Static_assert(c, m)
#endif
ET_B200_ABI_ASSERT(sizeof(void *) == 8u && sizeof(size_t) == 8u,
                   "K1 v1 needs 64-bit pointers and size_t");
ET_B200_ABI_ASSERT(sizeof(et_kernel_error) == 264u &&
                       offsetof(et_kernel_error, message) == 72u,
                   "K1 error record layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_dimension_range_v1) == 24u,
                   "K1 dimension range layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_shape_range_v1) == 16u,
                   "K1 shape range layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_capability_v1) == 120u &&
                       offsetof(et_kernel_capability_v1, shape_ranges) == 112u,
                   "K1 capability layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_tensor_view_v1) == 72u &&
                       offsetof(et_kernel_tensor_view_v1, shape) == 64u,
                   "K1 tensor view layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_request_v1) == 56u &&
                       offsetof(et_kernel_request_v1, deterministic) == 48u,
                   "K1 request layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_call_v1) == 88u &&
                       offsetof(et_kernel_call_v1, outputs) == 80u,
                   "K1 call layout");
ET_B200_ABI_ASSERT(sizeof(et_kernel_provider_v1) == 96u &&
                       offsetof(et_kernel_provider_v1, invoke_call) == 88u,
                   "K1 provider layout");
#undef ET_B200_ABI_ASSERT

#ifdef __cplusplus
}
#endif
#endif
