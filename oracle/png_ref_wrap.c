/* Test infrastructure only: the reference's PNG decode, compiled from the
 * reference's own vendored Wuffs (third_party/wuffs/wuffs-v0.4.c, included in
 * place, never copied) and driven exactly as
 * src/decode/fast_png_decoder.cpp:48-128 drives it:
 *   decode_image_config -> per-side cap (MAX_IMAGE_DIM) and pixel-area cap
 *   (MAX_IMAGE_PIXELS_MP, image_config.h:13-38) -> pixel buffer BGR,
 *   subsampling none -> decode_frame_config -> decode_frame with
 *   WUFFS_BASE__PIXEL_BLEND__SRC and a work buffer of workbuf_len().max_incl.
 * 16-bit PNGs take the reference's OpenCV route (fast_png_decoder.cpp:46-62);
 * that leg lives in the Python tests (cv2.imdecode), not here.
 * The caps are parameters so the tests can exercise the environment knobs. */
#define WUFFS_IMPLEMENTATION
#define WUFFS_CONFIG__STATIC_FUNCTIONS
#include "wuffs-v0.4.c"

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static _Thread_local const char *g_last = "";

const char *png_ref_last_status(void) { return g_last; }

/* 1 when the IHDR bit-depth byte says 16 (fast_png_decoder.cpp:24-26). */
int png_ref_is_16bit(const uint8_t *d, size_t len) {
  return len >= 26 && d[0] == 0x89 && d[1] == 'P' && d[2] == 'N' && d[3] == 'G' &&
         d[24] == 16;
}

/* Dimensions from Wuffs' image config; 0 on success. */
int png_ref_info(const uint8_t *data, size_t len, uint32_t *w, uint32_t *h) {
  wuffs_png__decoder dec;
  wuffs_base__status st = wuffs_png__decoder__initialize(&dec, sizeof dec, WUFFS_VERSION,
                                                         WUFFS_INITIALIZE__DEFAULT_OPTIONS);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -1; }
  wuffs_base__io_buffer src = wuffs_base__ptr_u8__reader((uint8_t *)data, len, true);
  wuffs_base__image_config ic;
  st = wuffs_png__decoder__decode_image_config(&dec, &ic, &src);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -2; }
  *w = wuffs_base__pixel_config__width(&ic.pixcfg);
  *h = wuffs_base__pixel_config__height(&ic.pixcfg);
  return 0;
}

/* Decode to BGR (w*h*3 bytes, tightly packed) into out (out_len bytes).
 * Returns 0 on success, 1 when the caps reject the image, negative when
 * Wuffs fails (the message is in png_ref_last_status). */
int png_ref_decode_bgr(const uint8_t *data, size_t len, uint32_t max_dim, int64_t max_pixels,
                       uint8_t *out, size_t out_len, uint32_t *w_out, uint32_t *h_out) {
  g_last = "";
  wuffs_png__decoder dec;
  wuffs_base__status st = wuffs_png__decoder__initialize(&dec, sizeof dec, WUFFS_VERSION,
                                                         WUFFS_INITIALIZE__DEFAULT_OPTIONS);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -1; }
  wuffs_base__io_buffer src = wuffs_base__ptr_u8__reader((uint8_t *)data, len, true);
  wuffs_base__image_config ic;
  st = wuffs_png__decoder__decode_image_config(&dec, &ic, &src);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -2; }
  uint32_t w = wuffs_base__pixel_config__width(&ic.pixcfg);
  uint32_t h = wuffs_base__pixel_config__height(&ic.pixcfg);
  *w_out = w;
  *h_out = h;
  if (w == 0 || h == 0 || w > max_dim || h > max_dim) return 1;
  if ((int64_t)w * (int64_t)h > max_pixels) return 1;
  size_t need = (size_t)w * h * 3;
  if (out_len < need) { g_last = "output buffer too small"; return -3; }

  wuffs_base__pixel_config pc;
  wuffs_base__pixel_config__set(&pc, WUFFS_BASE__PIXEL_FORMAT__BGR,
                                WUFFS_BASE__PIXEL_SUBSAMPLING__NONE, w, h);
  wuffs_base__slice_u8 pix = {out, need};
  wuffs_base__pixel_buffer pb;
  st = wuffs_base__pixel_buffer__set_from_slice(&pb, &pc, pix);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -4; }

  uint64_t wlen = wuffs_png__decoder__workbuf_len(&dec).max_incl;
  uint8_t *work = (uint8_t *)malloc(wlen ? wlen : 1);
  if (!work) { g_last = "out of memory"; return -5; }
  wuffs_base__slice_u8 ws = {work, (size_t)wlen};
  wuffs_base__frame_config fc;
  st = wuffs_png__decoder__decode_frame_config(&dec, &fc, &src);
  if (wuffs_base__status__is_ok(&st))
    st = wuffs_png__decoder__decode_frame(&dec, &pb, &src, WUFFS_BASE__PIXEL_BLEND__SRC, ws,
                                          NULL);
  free(work);
  if (!wuffs_base__status__is_ok(&st)) { g_last = st.repr; return -6; }
  return 0;
}
