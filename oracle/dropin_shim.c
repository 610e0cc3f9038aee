/* dropin_shim.c -- TEST INFRASTRUCTURE: the reference library with the B200
 * backend plugged in at its one dispatch point.
 *
 * `make -C oracle dropin REF_SRC=<reference>/bafe` compiles the reference's
 * own, unmodified src/*.c and links them with this file into
 * oracle/_ref/libbafe_dropin.so.  Only jit.c is compiled differently: with
 * -Dbafe_jit_get_or_compile=bafe_jit_get_or_compile_c99, so its definition
 * (jit.c:204) and its declaration (jit.h:45-46) take that name, and every
 * other caller in the library -- bafe_optimize_and_compile[_with_budget]
 * (bafe.c:260-279) and bafe_fuse_compile (fuse.c:109-125) -- reaches the
 * dispatch below instead.  This is the switch a maintainer adds at the top of
 * jit.c's bafe_jit_get_or_compile (the recipe is the C side of the
 * integration notes): BAFE_BACKEND=cuda routes the graph to
 * bafe_cuda_jit_get_or_compile from libbafe_cuda.so, anything else keeps the
 * reference's C99 emitter.
 */
#include <stdlib.h>
#include <string.h>

#include "bafe/jit.h"          /* the reference's bafe_graph and bafe_kernel_fn */

bafe_kernel_fn bafe_jit_get_or_compile_c99(const bafe_graph *g, char *err_buf, size_t err_buf_size);

/* include/bafe_cuda.h:177 -- declared here rather than by including that
 * header, so the reference's own type definitions are the only ones in
 * this translation unit (the header's copies are layout-identical). */
bafe_kernel_fn bafe_cuda_jit_get_or_compile(const bafe_graph *g, char *err_buf, size_t err_buf_size);

bafe_kernel_fn bafe_jit_get_or_compile(const bafe_graph *g, char *err_buf, size_t err_buf_size) {
    const char *backend = getenv("BAFE_BACKEND");
    if (backend && strcmp(backend, "cuda") == 0)
        return bafe_cuda_jit_get_or_compile(g, err_buf, err_buf_size);
    return bafe_jit_get_or_compile_c99(g, err_buf, err_buf_size);
}
