/* Plain-C client of include/cpg.h, as the reference's C11 engine would be: compiled with gcc
 * -std=c11 and linked against libcpg_b200.so. Calls only entry points that fail or finish
 * before any CUDA work, so it runs without a GPU. Prints "ok" on success. */
#include <stdio.h>
#include <string.h>

#include "cpg.h"

int main(void) {
    if (cpg_version() != 100) { puts("version"); return 1; }
    if (cpg_dequant(NULL, NULL, CPG_ENC_Q4, 64, NULL) != CPG_EINVAL) { puts("dequant"); return 1; }
    if (strstr(cpg_last_error(), "null") == NULL) { puts("last_error"); return 1; }
    if (cpg_store_add_region(0, 16, 1) != CPG_ESTATE) { puts("store"); return 1; }
    if (cpg_store_verify(NULL, 0, NULL) != CPG_ESTATE) { puts("verify"); return 1; }
    uint32_t crc = 7;
    if (cpg_crc32(NULL, 0, &crc, NULL) != CPG_OK || crc != 0u) { puts("crc32"); return 1; }
    int st[3];
    double er[2];
    if (cpg_route_check(NULL, NULL, NULL, 0, 128, 8, st, er, NULL) != CPG_OK || st[2] != -1) { puts("route"); return 1; }
    cpg_moe_desc d;
    memset(&d, 0, sizeof d);
    cpg_moe_layer *L = NULL;
    if (cpg_moe_layer_create(&d, &L) != CPG_EINVAL || L != NULL) { puts("layer"); return 1; }
    puts("ok");
    return 0;
}
