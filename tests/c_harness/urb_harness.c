/* urb_harness.c — drives the C ABI exactly as a Rust crate's build.rs links it: liburb_moe.a +
 * the static CUDA runtime + libstdc++ / rt / pthread / dl, no Python in the process.
 *
 *   urb_harness <input.bin> <output.bin>
 *
 * input.bin (little endian): u32 hidden, inter, experts, top_k, tokens; f32 routed scale;
 * router bf16 bits [experts, hidden]; bias f32 [experts]; for each of the experts + 1 gated
 * MLPs (the shared expert last) MXFP4 gate, up [inter, hidden] and down [hidden, inter], each
 * as packed nibbles [rows, cols/2] then E8M0 scales [rows, cols/32]; x f32 [tokens, hidden].
 * output.bin: out f32 [tokens, hidden], route experts i32 [tokens, top_k], route weights f32
 * [tokens, top_k], then y f32 [64] = rows 5..68 of expert 0's gate times x[0]
 * (WeightMatrix::matvec_rows).
 *
 * Calls: urb_ctx_create -> urb_mxfp4_upload / urb_bf16_upload -> urb_moe_layer_create ->
 * urb_moe_forward (RuntimeMoeLayer::forward, src/models/glm/runtime/moe.rs:138) ->
 * urb_matvec_rows -> urb_last_error on a rejected upload (a 0xFF scale: MxError::InvalidScale)
 * -> frees.  Exit status 0 and "OK" on success. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "urb_moe.h"

static urb_ctx *g_ctx;

static void die(const char *what, int rc) {
    char msg[512] = {0};
    if (g_ctx) urb_last_error(g_ctx, msg, sizeof msg);
    fprintf(stderr, "%s failed: status %d: %s\n", what, rc, msg);
    exit(1);
}

static void *read_n(FILE *f, size_t bytes) {
    void *p = malloc(bytes ? bytes : 1);
    if (!p || fread(p, 1, bytes, f) != bytes) {
        fprintf(stderr, "short input\n");
        exit(1);
    }
    return p;
}

static urb_mat *mxfp4(FILE *f, size_t rows, size_t cols) {
    const size_t np = rows * (cols / 2), ns = rows * (cols / 32);
    uint8_t *packed = read_n(f, np), *scales = read_n(f, ns);
    urb_mat *m = NULL;
    int rc = urb_mxfp4_upload(g_ctx, rows, cols, 32, packed, np, scales, ns, &m);
    if (rc) die("urb_mxfp4_upload", rc);
    free(packed);
    free(scales);
    return m;
}

int main(int argc, char **argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s input.bin output.bin\n", argv[0]);
        return 2;
    }
    FILE *f = fopen(argv[1], "rb");
    if (!f) return 2;
    uint32_t hdr[5];
    float scale;
    if (fread(hdr, 4, 5, f) != 5 || fread(&scale, 4, 1, f) != 1) return 2;
    const size_t H = hdr[0], I = hdr[1], E = hdr[2], K = hdr[3], T = hdr[4];
    int rc = urb_ctx_create(0, &g_ctx);
    if (rc) die("urb_ctx_create", rc);

    uint16_t *router_bits = read_n(f, E * H * 2);
    float *bias = read_n(f, E * 4);
    urb_mat *router = NULL;
    rc = urb_bf16_upload(g_ctx, E, H, router_bits, E * H, &router);
    if (rc) die("urb_bf16_upload", rc);
    urb_mat **gate = calloc(E + 1, sizeof *gate), **up = calloc(E + 1, sizeof *up),
            **down = calloc(E + 1, sizeof *down);
    for (size_t e = 0; e <= E; ++e) {
        gate[e] = mxfp4(f, I, H);
        up[e] = mxfp4(f, I, H);
        down[e] = mxfp4(f, H, I);
    }
    float *x = read_n(f, T * H * 4);
    fclose(f);

    const urb_moe_geometry geo = {(uint32_t)K, 1, 1, 1, scale};
    urb_layer *layer = NULL;
    rc = urb_moe_layer_create(g_ctx, router, bias, E, (const urb_mat *const *)gate,
                              (const urb_mat *const *)up, (const urb_mat *const *)down, gate[E],
                              up[E], down[E], &geo, &layer);
    if (rc) die("urb_moe_layer_create", rc);
    float *out = malloc(T * H * 4), *w = malloc(T * K * 4), y[64];
    int32_t *ids = malloc(T * K * 4);
    rc = urb_moe_forward(g_ctx, layer, x, T, out, ids, w, NULL, NULL, NULL, NULL, NULL);
    if (rc) die("urb_moe_forward", rc);
    rc = urb_matvec_rows(g_ctx, gate[0], 5, 64, x, H, y);
    if (rc) die("urb_matvec_rows", rc);

    /* A rejected upload reports MxError::InvalidScale and leaves a message. */
    uint8_t bad_packed[16] = {0}, bad_scales[1] = {0xFF};
    urb_mat *bad = NULL;
    rc = urb_mxfp4_upload(g_ctx, 1, 32, 32, bad_packed, 16, bad_scales, 1, &bad);
    char msg[256] = {0};
    if (rc != URB_ERR_INVALID_SCALE || urb_last_error(g_ctx, msg, sizeof msg) != URB_ERR_INVALID_SCALE ||
        msg[0] == 0) {
        fprintf(stderr, "0xFF scale: status %d, message '%s'\n", rc, msg);
        return 1;
    }

    FILE *o = fopen(argv[2], "wb");
    if (!o || fwrite(out, 4, T * H, o) != T * H || fwrite(ids, 4, T * K, o) != T * K ||
        fwrite(w, 4, T * K, o) != T * K || fwrite(y, 4, 64, o) != 64)
        return 2;
    fclose(o);

    urb_moe_layer_free(layer);
    for (size_t e = 0; e <= E; ++e) {
        urb_mat_free(gate[e]);
        urb_mat_free(up[e]);
        urb_mat_free(down[e]);
    }
    urb_mat_free(router);
    rc = urb_ctx_destroy(g_ctx);
    if (rc) return 1;
    printf("OK\n");
    return 0;
}
