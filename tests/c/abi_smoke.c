/* A C caller of the library (no C++, no torch): checks the ABI version against the header
 * and calls entry points that need no GPU (argument errors, workspace sizes). */
#include <stdio.h>
#include <string.h>

#include "b200_attn.h"

int main(void) {
    if (b200_abi_version() != B200_ABI_VERSION) {
        printf("ABI version %d, header %d\n", b200_abi_version(), B200_ABI_VERSION);
        return 1;
    }
    /* a null cache pointer is an argument error, reported before any CUDA call */
    int32_t rc = b200_store_kvcache(NULL, 1024, NULL, 1024, NULL, NULL, NULL, 4, 8, 128, 1024, 2, NULL);
    if (rc != B200_ERR_ARG || strstr(b200_last_error(), "null") == NULL) {
        printf("store_kvcache: rc %d, '%s'\n", rc, b200_last_error());
        return 2;
    }
    size_t ws = b200_paged_attention_workspace_size(1000, 1, 2, 128);
    size_t ws2 = b200_paged_attention_workspace_size(2000, 1, 2, 128);
    if (ws == 0 || ws % 256 != 0 || ws2 <= ws) {
        printf("paged workspace sizes %zu %zu\n", ws, ws2);
        return 3;
    }
    /* an output size the fused o_proj kernel does not tile */
    char dummy[16];
    void* slots[1] = {dummy};
    uint32_t* flags[1] = {(uint32_t*)dummy};
    rc = b200_oproj_allreduce(dummy, 300, dummy, 64, dummy, 64, 8, 300, 64, slots, 8, NULL, 0, flags, 1, NULL, 0,
                              0, 1, NULL);
    if (rc != B200_ERR_UNSUPPORTED) {
        printf("oproj_allreduce: rc %d, '%s'\n", rc, b200_last_error());
        return 4;
    }
    printf("ok abi %d, paged workspace %zu bytes for 1000 items\n", b200_abi_version(), ws);
    return 0;
}
