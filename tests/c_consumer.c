/* A plain C99 host of the C ABI: includes include/hilberta_b200.h, links
 * libhilberta_b200.so and calls the entry points' host-side paths (no GPU):
 * version and status strings, plan dimensions, workspace sizes and argument
 * checks that return before any launch.  Prints "ok" and exits 0 on success. */
#include <stdio.h>
#include <string.h>

#include "hilberta_b200.h"

#define CHECK(cond)                                                  \
    do {                                                             \
        if (!(cond)) {                                               \
            fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            return 1;                                                \
        }                                                            \
    } while (0)

int main(void) {
    CHECK(hb_version() >= 100);
    CHECK(strcmp(hb_status_string(HB_OK), "ok") == 0);
    hb_plan_dims_t d;
    CHECK(hb_plan_dims(128, 16, 512, 64, 0, &d) == HB_OK);
    CHECK(d.image_tokens == 16384 && d.total_blocks == 264 && d.rows == 256);
    CHECK(hb_plan_dims(12, 4, 512, 64, 0, &d) == HB_ERR_ARG);
    CHECK(hb_fwd_workspace_bytes() >= 12);
    CHECK(hb_fwd_workspace_bytes_for(1, 24, 16896, 512, 128) > hb_fwd_workspace_bytes());
    /* argument checks that return before touching a device */
    int32_t dummy[4];
    CHECK(hb_expand_kv128(dummy, dummy, 4, 0, dummy, 1, dummy, dummy, 8, dummy, NULL) == HB_ERR_ARG);
    CHECK(hb_expand_kv128(NULL, NULL, 4, 4, NULL, 0, NULL, NULL, 8, NULL, NULL) == HB_OK);
    CHECK(hb_adaln_residual(NULL, 3072, NULL, 0, NULL, NULL, NULL, 0, NULL, 0, NULL, 0, 16, 16, 3072, 1e-6f, 1,
                            NULL) == HB_ERR_ARG);
    CHECK(hb_adaln_residual(dummy, 128, NULL, 0, NULL, dummy, dummy, 0, NULL, 0, dummy, 128, 16, 16, 128, 1e-6f, 1,
                            NULL) == HB_ERR_UNSUPPORTED);
    puts("ok");
    return 0;
}
