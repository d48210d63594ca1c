/* SPDX-License-Identifier: Unlicense */

/* Weight files of the B200 build: the reference's pth_loader.h API
 * (pth_loader.h:38-61 of i.coregistration.opencl) over the formats the
 * reference reads: torch.save zip archives (stored entries, zip64 aware),
 * the legacy torch.save stream, and safetensors. The state_dict is the
 * saved dict, or its "model" / "state_dict" entry, or its only dict of
 * tensors; float32, float16 and bfloat16 tensors are indexed (views keep
 * their strides and storage offsets), other dtypes are left out. Errors go
 * through the library's fatal / recording mode (ocl_backend.h).
 *
 *   pth_open          replaces pth_loader.c:1148
 *   pth_find          replaces pth_loader.c:1228
 *   pth_require       replaces pth_loader.c:1254
 *   pth_strip_prefix  replaces pth_loader.c:1238
 *   pth_numel         replaces pth_loader.c:1275
 *   pth_bytes         replaces pth_loader.c:1379
 *   pth_read_f32      replaces pth_loader.c:1330 (F32 / F16 / BF16 -> F32,
 *                     strided views gathered in C order)
 *   pth_close         replaces pth_loader.c:1392 */

#ifndef I_COREGISTRATION_B200_PTH_LOADER_H
#define I_COREGISTRATION_B200_PTH_LOADER_H

#include <stdio.h>
#include <sys/types.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PTH_MAX_DIMS 8

enum pth_dtype { PTH_F32, PTH_F16, PTH_BF16, PTH_OTHER };

struct pth_tensor {
    char *name;
    int ndim;
    long shape[PTH_MAX_DIMS];
    long stride[PTH_MAX_DIMS];
    long storage_offset; /* In elements. */
    enum pth_dtype dtype;
    off_t data_offset;    /* Byte offset of the data in the file. */
    size_t storage_bytes; /* Byte size of the data. */
};

struct pth_file {
    FILE *fp;
    char *path;
    int ntensors;
    struct pth_tensor *tensors;
};

void pth_open(struct pth_file *pf, const char *path);
const struct pth_tensor *pth_find(const struct pth_file *pf, const char *name);
const struct pth_tensor *pth_require(const struct pth_file *pf,
                                     const char *name, int ndim,
                                     const long *shape);
int pth_strip_prefix(struct pth_file *pf, const char *prefix);
long pth_numel(const struct pth_tensor *t);
double pth_bytes(const struct pth_file *pf, const char *prefix);
float *pth_read_f32(const struct pth_file *pf, const struct pth_tensor *t);
void pth_close(struct pth_file *pf);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_PTH_LOADER_H */
