/* libsplat_b200 — the splat file formats around the path: the binary PLY of the 3DGS
 * reference implementation (instantsplat-rs/src/splat_ply.rs), read and written from and to
 * the packed parameter layout the kernels use, on the host or straight from device memory.
 *
 * Layout of a written file: the reference's header ("ply", "format binary_little_endian
 * 1.0", a comment, "element vertex N", one "property float" line per value, "end_header"),
 * then N little-endian float records. At SH degree 0 the properties are the reference's 17,
 * in its order (splat_ply.rs:12-16): x y z nx ny nz f_dc_0..2 opacity scale_0..2 rot_0..3,
 * normals written as 0. At SH degrees 1-3 the 3DGS convention adds f_rest_0 ..
 * f_rest_{3(K-1)-1} after f_dc (K = (degree + 1)^2 coefficients, channel-major: f_rest_{c (K-1)
 * + k - 1} is coefficient k of channel c), which the reference's writer does not produce and
 * its reader skips.
 *
 * Reading accepts what the reference's parser accepts (splat_ply.rs:54-112): float
 * properties in any order, comments, extra properties skipped; and refuses what it refuses,
 * with its messages (sp_ply_error): not a PLY file, a header that never ends, another
 * element, a non-float property, an unexpected header line, no vertex element, a missing
 * property, a short file.
 */
#ifndef SPLAT_IO_H
#define SPLAT_IO_H

#include <stdint.h>

#include "splat.h"

#ifdef __cplusplus
extern "C" {
#endif

/* write_splat_ply (splat_ply.rs:18-46) of `count` Gaussians packed at `sh_degree` (stride
 * 11 + 3 (degree + 1)^2). `params` is host memory, or device memory when params_on_device
 * is 1 (copied to the host in one transfer). SP_ERR_INVALID with a message (sp_ply_error)
 * when the file cannot be written. */
sp_status sp_ply_write(const char* path, const float* params, uint64_t count, uint32_t sh_degree,
                       int params_on_device);

/* The vertex count of a splat PLY and the SH degree its f_rest_* properties carry (0 when it
 * has none; 1-3 for 9, 24 or 45 of them). */
sp_status sp_ply_read_header(const char* path, uint64_t* count, uint32_t* sh_degree);

/* read_splat_ply (splat_ply.rs:48-112) into `count` Gaussians packed at `sh_degree` (host
 * memory, or device memory with params_on_device = 1). A degree below the file's drops the
 * higher coefficients (degree 0 is the reference's reader); one above it zeroes them.
 * `count` must be the file's. */
sp_status sp_ply_read(const char* path, float* params, uint64_t count, uint32_t sh_degree, int params_on_device);

/* The message of the last sp_ply_* failure on this thread. */
const char* sp_ply_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SPLAT_IO_H */
