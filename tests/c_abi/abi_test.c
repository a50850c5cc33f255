/* A C caller of libsplat_b200 (no GPU needed): what a Rust FFI binding of include/splat.h
 * and include/splat_io.h does, in C. Exercises the host-only entry points: version and
 * status strings, the densify schedule, the position-rate decay, a PLY written and read
 * back, and the argument checks that stand in for the reference's panics. Prints "ok" and
 * exits 0, or names the first failed check and exits 1. */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "splat.h"
#include "splat_constants.h"
#include "splat_io.h"

#define CHECK(cond)                                              \
    do {                                                         \
        if (!(cond)) {                                           \
            fprintf(stderr, "failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                            \
        }                                                        \
    } while (0)

int main(int argc, char** argv) {
    const char* path = argc > 1 ? argv[1] : "abi_test.ply";
    CHECK(sp_version() != NULL && strlen(sp_version()) > 0);
    CHECK(sp_status_string(SP_OK) != NULL);
    /* The struct layouts a Rust #[repr(C)] binding mirrors. */
    CHECK(sizeof(sp_options) == 36 && sizeof(sp_densify_settings) == 40 && sizeof(sp_densify_report) == 64);
    CHECK(sizeof(sp_camera_uniform) == 80 && sizeof(sp_densify_stats) == 16);
    sp_options defaults;
    sp_options_default(&defaults);
    CHECK(defaults.tile_culling == SP_TILES_RECTANGLE && defaults.intersections_per_gaussian == 24);

    /* DENSIFY_SHORT_RUN (densify.rs:59-69): densified after 50, 100, 150 of 300 steps. */
    sp_densify_settings s = {50, 50, 0.5f, 2e-4f, 0.01f, 0.005f, 100.0f, 2.0f, 0, 0};
    int after[8], found = 0;
    for (uint64_t done = 1; done <= 300; ++done) {
        const int due = sp_densify_after(&s, done, 300);
        CHECK(due == 0 || due == 1);
        if (due && found < 8) after[found++] = (int)done;
    }
    CHECK(found == 3 && after[0] == 50 && after[1] == 100 && after[2] == 150);
    CHECK(sp_densify_after(&s, 0, 300) == -1 && sp_densify_after(&s, 301, 300) == -1);
    s.opacity_reset_interval = 75;
    CHECK(sp_resets_opacity_after(&s, 150) == -1);
    s.opacity_reset_interval = 100;
    CHECK(sp_resets_opacity_after(&s, 100) == 1 && sp_resets_opacity_after(&s, 50) == 0);

    /* position_rate_factor (optimizer.rs:59-62): 1 at the first step, 0.01 at the last. */
    CHECK(sp_position_rate_factor(0, 100) == 1.0f);
    CHECK(fabsf(sp_position_rate_factor(99, 100) - 0.01f) < 1e-7f);
    CHECK(sp_position_rate_factor(100, 100) < 0.0f);

    /* A PLY round trip at SH degree 1 (stride 23). */
    enum { N = 3, STRIDE = SP_PARAM_STRIDE(1) };
    float params[N * STRIDE], back[N * STRIDE];
    for (int i = 0; i < N * STRIDE; ++i) params[i] = 0.25f * (float)i - 3.0f;
    CHECK(sp_ply_write(path, params, N, 1, 0) == SP_OK);
    uint64_t count = 0;
    uint32_t degree = 9;
    CHECK(sp_ply_read_header(path, &count, &degree) == SP_OK && count == N && degree == 1);
    CHECK(sp_ply_read(path, back, N, 1, 0) == SP_OK);
    CHECK(memcmp(params, back, sizeof(params)) == 0);
    CHECK(sp_ply_read(path, back, N + 1, 1, 0) == SP_ERR_INVALID && strlen(sp_ply_error()) > 0);

    /* Null handles are refused, not dereferenced. */
    CHECK(sp_forward(NULL) == SP_ERR_INVALID);
    CHECK(sp_adam_step(NULL, 1.0f) == SP_ERR_INVALID);
    CHECK(sp_densify_apply(NULL, NULL, NULL, NULL, 0) == SP_ERR_INVALID);
    CHECK(sp_peer_export(NULL, NULL) == SP_ERR_INVALID && sp_peer_exchange_step(NULL, 1.0f) == SP_ERR_INVALID);
    CHECK(sizeof(sp_peer_handle) == 160);
    printf("ok\n");
    return 0;
}
