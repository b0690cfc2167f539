/* rad_encoding.h -- the encoding half of the radiance engine's plugin ABI (ABI 17), restated: how a
 * quantised weight names its scheme, transform and planes, and what a row's layout hook answers.
 *
 * Declares what include/exl3_encoding.h:84-126 (exl3_encoding_make / _read), kernels/exl3ref/ref.c:180
 * (rad_enc_row_bytes) and kernels/exl3r4d/layout.c use. Source-compatible by construction. */
#ifndef RAD_ENCODING_H
#define RAD_ENCODING_H

#include "rad_types.h"

#ifdef __cplusplus
extern "C" {
#endif

#define RAD_ENC_STR 32
#define RAD_ENC_MAX_PLANES 8
/* The engine's default alignment of a stored weight, and of a sub-plane inside a unit. */
#define RAD_ALIGN_UNIT 4096
#define RAD_ALIGN_SUB 256

typedef struct RadEncPlane {
    char     name[RAD_ENC_STR];
    uint32_t dtype;
    int32_t  tile_r, tile_c;   /* the TILED [r x c] cut rule; 0 = the whole extent */
} RadEncPlane;

typedef struct RadEncoding {
    char        scheme[RAD_ENC_STR];
    char        transform[RAD_ENC_STR];
    int32_t     n_planes;
    RadEncPlane plane[RAD_ENC_MAX_PLANES];
} RadEncoding;

/* A row's answer to "how will you store this plane": the stored type, its bytes and alignment, and a tag
 * naming the form. */
typedef struct RadLayout {
    uint32_t    dtype;
    int64_t     bytes;
    int64_t     align;
    const char* tag;
} RadLayout;

static inline void rad_enc_clear(RadEncoding* e) { memset(e, 0, sizeof *e); }
static inline void rad_enc_copy_str(char* dst, const char* src) {
    size_t n = src ? strlen(src) : 0;
    if (n >= RAD_ENC_STR) n = RAD_ENC_STR - 1;
    memset(dst, 0, RAD_ENC_STR);
    if (n) memcpy(dst, src, n);
}
static inline int rad_enc_add_plane(RadEncoding* e, const char* name, uint32_t dtype, int tile_r, int tile_c) {
    if (!e || e->n_planes >= RAD_ENC_MAX_PLANES) return RAD_E_SHAPE;
    RadEncPlane* p = &e->plane[e->n_planes++];
    rad_enc_copy_str(p->name, name);
    p->dtype = dtype;
    p->tile_r = tile_r;
    p->tile_c = tile_c;
    return RAD_OK;
}
static inline int rad_enc_is(const RadEncoding* e, const char* scheme) {
    return e && scheme && strncmp(e->scheme, scheme, RAD_ENC_STR) == 0;
}
static inline int rad_enc_equal(const RadEncoding* a, const RadEncoding* b) {
    return a && b && memcmp(a, b, sizeof *a) == 0;
}
/* Bytes of one row of `cols` elements of `dtype`, each row starting on a byte. */
static inline int64_t rad_enc_row_bytes(uint32_t dtype, int64_t cols) { return rad_dtype_bytes(dtype, cols); }

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* RAD_ENCODING_H */
