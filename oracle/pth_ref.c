/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's checkpoint reader (pth_loader.c),
 * compiled where it lies (the Makefile names it by path in
 * REF_PTH_LOADER_C), the checker of this build's pth_loader. Its entry
 * points (pth_open, pth_find, pth_read_f32, pth_bytes, pth_close ...) are
 * exported as they are; the progress meter it feeds is a no-op here.
 * Every failure exits the process (G_fatal_error), so it is only given
 * well-formed files. Built into _ref/libpth_ref.so by oracle/Makefile. */

#include REF_PTH_LOADER_C

void progress_bytes(size_t n) { (void)n; }
