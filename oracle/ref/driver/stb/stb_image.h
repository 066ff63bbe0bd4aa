/*
 * stb_image-compatible loader for building the reference's benchmark driver
 * against libnerf_b200.so (test infrastructure only).  The driver calls
 * stbi_load(path, &w, &h, &channels, 4) and stbi_image_free(pixels); this
 * header provides those two entry points over the library's own PNG decoder
 * (nerf_b200_png_read), so no third-party image library is needed.  Only
 * desired_channels == 4 (RGBA8) is supported, which is what the driver asks
 * for.  STB_IMAGE_IMPLEMENTATION, which the driver defines, is ignored.
 */
#ifndef NERF_B200_STB_IMAGE_SHIM_H
#define NERF_B200_STB_IMAGE_SHIM_H

#include <stdint.h>
#include <stdlib.h>

#include "nerf_b200.h"

typedef unsigned char stbi_uc;

static inline stbi_uc* stbi_load(char const* filename, int* x, int* y, int* channels_in_file, int desired_channels) {
    uint32_t w = 0, h = 0;
    if (!filename || desired_channels != 4) return NULL;
    if (nerf_b200_png_read(filename, NULL, 0, &w, &h) != NERF_STATUS_OK || w == 0 || h == 0) return NULL;
    const uint64_t bytes = (uint64_t)w * h * 4u;
    stbi_uc* out = (stbi_uc*)malloc(bytes);
    if (!out) return NULL;
    if (nerf_b200_png_read(filename, out, bytes, &w, &h) != NERF_STATUS_OK) {
        free(out);
        return NULL;
    }
    if (x) *x = (int)w;
    if (y) *y = (int)h;
    if (channels_in_file) *channels_in_file = 4;
    return out;
}

static inline void stbi_image_free(void* retval_from_stbi_load) { free(retval_from_stbi_load); }

#endif
