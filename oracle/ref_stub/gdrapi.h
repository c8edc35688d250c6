/* TEST INFRASTRUCTURE ONLY: declarations of the GDRCopy user-API calls the
 * reference's search backends make, so that their device code can be compiled
 * in place for oracle/ref_kernels.cu without the GDRCopy library.  The
 * harness defines these to fail; it only launches the device-resident
 * kernels, which never touch a GDRCopy mapping. */
#ifndef GOFANN_REF_STUB_GDRAPI_H
#define GOFANN_REF_STUB_GDRAPI_H
#include <stddef.h>
#include <stdint.h>
typedef struct gofann_ref_gdr_stub* gdr_t;
typedef struct {
    unsigned long h;
} gdr_mh_t;
#ifdef __cplusplus
extern "C" {
#endif
gdr_t gdr_open(void);
int gdr_close(gdr_t g);
int gdr_pin_buffer(gdr_t g, unsigned long addr, size_t size, uint64_t p2p_token, uint32_t va_space, gdr_mh_t* handle);
int gdr_unpin_buffer(gdr_t g, gdr_mh_t handle);
int gdr_map(gdr_t g, gdr_mh_t handle, void** va, size_t size);
int gdr_unmap(gdr_t g, gdr_mh_t handle, void* va, size_t size);
#ifdef __cplusplus
}
#endif
#endif
