/* Opaque Level Zero handle types, and nothing else.
 *
 * The reference's qwen3/level_zero_runtime.hpp includes <level_zero/ze_api.h>
 * only to declare its private handle members. With this directory on the
 * include path that header compiles unchanged on a machine without Level
 * Zero, and the CUDA implementation in host/qwen3/level_zero_runtime_cuda.cpp
 * provides its methods (it never uses these members). */
#ifndef XPU_ZE_SHIM_ZE_API_H
#define XPU_ZE_SHIM_ZE_API_H

typedef struct _ze_driver_handle_t *ze_driver_handle_t;
typedef struct _ze_device_handle_t *ze_device_handle_t;
typedef struct _ze_context_handle_t *ze_context_handle_t;
typedef struct _ze_command_list_handle_t *ze_command_list_handle_t;
typedef struct _ze_module_handle_t *ze_module_handle_t;
typedef struct _ze_kernel_handle_t *ze_kernel_handle_t;

#endif
