/* A plain C11 consumer of the drop-in boundary: it includes the public
 * headers, checks the reference ABI's struct layouts at compile time
 * (qw35-server/src/metal/bridge/Qw35MetalTypes.h:9-66, LP64), links against
 * libqw35cuda.so and calls the entry points that need no GPU.  Built and run
 * by tests/test_boundary.py. */
#include <stddef.h>
#include <stdio.h>
#include <string.h>

#include "qw35_cuda.h"
#include "qw35_ffi.h"

_Static_assert(sizeof(qw35_metal_tensor_desc) == 80, "tensor desc size");
_Static_assert(offsetof(qw35_metal_tensor_desc, abs_offset) == 56, "tensor desc abs_offset");
_Static_assert(offsetof(qw35_metal_hparams, n_cls_out) == sizeof(qw35_metal_hparams) - 4, "hparams tail");
_Static_assert(sizeof(qw35_metal_warm_report) == 48, "warm report size");

static int fail(const char *what) {
    fprintf(stderr, "FAIL: %s\n", what);
    return 1;
}

int main(void) {
    char err[256];
    if (qw35_cuda_weight_bytes(QW35_TYPE_GF4, 12288, 4096) != 25165824ull) return fail("gf4 bytes");
    if (qw35_cuda_weight_bytes(QW35_TYPE_Q6_K, 248320, 4096) != 248320ull * 16 * 210) return fail("q6_k bytes");
    if (qw35_cuda_device_bytes(QW35_TYPE_Q8_0, 12288, 4096) != 53477376ull + 12288) return fail("q8_0 device bytes");
    memset(err, 'x', sizeof err);
    if (qw35_metal_runtime_sync((void *)0x1234, err, sizeof err) != 0) return fail("bogus handle accepted");
    if (strstr(err, "invalid qw35 runtime handle") == NULL) return fail("bogus handle message");
    if (qw35_cuda_matvec(7, (void *)1, (void *)1, 0, (float *)1, 16, 256, 1, 0, 0, NULL, err, sizeof err) != 0)
        return fail("unsupported type accepted");
    if (strstr(err, "unsupported weight type") == NULL) return fail("unsupported type message");
    puts("abi ok");
    return 0;
}
