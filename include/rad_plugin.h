/* rad_plugin.h -- a kernel plugin's identity and the symbols the radiance engine's loader resolves, restated
 * for ABI 17 from kernels/exl3ref/rows.c:243-258 and kernels/exl3r4d/rows.c:524-550.
 *
 * A kernel library exports (extern "C", resolved by dlsym):
 *   uint32_t             rad_plugin_abi_version(void);     == RAD_ABI_VERSION
 *   const RadPluginInfo* rad_plugin_info(void);
 *   int                  rad_kernel_schema_count(void);    the op schemas it implements
 *   const RadOpSchema*   rad_kernel_schema_at(int i);
 *   int                  rad_kernel_count(void);           its rows
 *   const RadKernelInfo* rad_kernel_at(int i);
 *   int                  rad_kernel_concurrent(int i);     optional: row i may run concurrently with itself
 *   int                  rad_plugin_reference(void);       optional: 1 for a reference library */
#ifndef RAD_PLUGIN_H
#define RAD_PLUGIN_H

#include "rad_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { RAD_PLUGIN_KERNEL = 1, RAD_PLUGIN_QUANT = 2, RAD_PLUGIN_ARCH = 3 };

typedef struct RadPluginInfo {
    int32_t     kind;          /* RAD_PLUGIN_* */
    const char* name;
    const char* version;
    const char* description;
    const char* target;        /* "host", or the device target the code is built for */
} RadPluginInfo;

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* RAD_PLUGIN_H */
