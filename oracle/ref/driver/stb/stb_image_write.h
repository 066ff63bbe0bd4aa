/*
 * stb_image_write-compatible PNG writer for building the reference's
 * benchmark driver against libnerf_b200.so (test infrastructure only): the
 * driver's stbi_write_png(path, w, h, 4, rgba, w * 4) goes to the library's
 * own encoder (nerf_b200_png_write, RGBA8).  Other channel counts or row
 * strides return 0 (failure).  STB_IMAGE_WRITE_IMPLEMENTATION is ignored.
 */
#ifndef NERF_B200_STB_IMAGE_WRITE_SHIM_H
#define NERF_B200_STB_IMAGE_WRITE_SHIM_H

#include <stdint.h>

#include "nerf_b200.h"

static inline int stbi_write_png(char const* filename, int w, int h, int comp, const void* data, int stride_in_bytes) {
    if (!filename || !data || w <= 0 || h <= 0 || comp != 4 || stride_in_bytes != w * 4) return 0;
    return nerf_b200_png_write(filename, (const uint8_t*)data, (uint32_t)w, (uint32_t)h) == NERF_STATUS_OK ? 1 : 0;
}

#endif
