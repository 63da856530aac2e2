// PNG decode on the device: a batch of PNG files already in HBM becomes
// BGR u8 HWC images (the reference's GpuImage layout), replacing the
// reference's CPU decode + upload (src/decode/fast_png_decoder.cpp:48-128,
// Wuffs v0.4 to a BGR cv::Mat, then OcrPipeline::upload_image,
// src/pipeline/ocr/ocr_pipeline_runtime.cpp:120-147).
//
// Three kernels:
//   png_parse_kernel    signature, IHDR, the chunks before the image data
//                       (PLTE / tRNS rules as Wuffs applies them), CRC-32 of
//                       every critical chunk (the warp splits a chunk into
//                       256-byte pieces and combines their CRCs with the
//                       x^(8n) mod P shift), a 64-byte record per image.
//   png_inflate_kernel  zlib header, DEFLATE (stored / fixed / dynamic
//                       blocks, RFC 1951), two warps per image: the decoder
//                       warp's lane 0 turns Huffman symbols into batches of
//                       tokens while the copier warp applies the previous
//                       batch to a 32 KB window in shared memory (literal
//                       runs and matches 32 bytes at a time); every 4 KB of
//                       window goes to the scanline buffer in HBM with
//                       16-byte stores and into the Adler-32.
//   png_unfilter_kernel the five PNG filters over a wavefront: lane k owns
//                       row r0 + k and runs one filter unit behind lane k-1,
//                       so the row above (b) and its left neighbour (c) come
//                       from lane k-1 by shuffle; one CTA per image, eight
//                       warps on consecutive groups of 32 rows, tiles staged
//                       in shared memory; colour conversion to BGR in the
//                       same pass (Wuffs' rules for 1-8 bit depths, OpenCV's
//                       for 16 bit, which is the decoder the reference
//                       routes 16-bit files to).
// Every loop is bounded by the input or output size. The waits between
// warps are a named barrier that both warps of an image reach once per batch
// (the same count on every path) and, in the unfilter, a spin on a
// shared-memory counter with an iteration limit (TOCR_PNG_TIMEOUT).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "tocr_common.cuh"

namespace tocr {
namespace png {

// ---- status codes (tocr_capi.h: TOCR_PNG_*) ----
enum : int32_t {
  kOk = 0,
  kBadHeader = 1,
  kBadChunk = 2,
  kBadChecksum = 3,
  kMissingPalette = 4,
  kBadZlib = 5,
  kBadDeflate = 6,
  kTooMuchData = 7,
  kNotEnoughData = 8,
  kBadFilter = 9,
  kSizeMismatch = 10,
  kUnsupported = 11,
  kTimeout = 12,
};

constexpr uint32_t kCrcPoly = 0xEDB88320u;  // CRC-32 (ISO-HDLC), reflected
constexpr int kMetaBytes = 64;

// Per-image scratch, from scratch_off (16-byte aligned):
//   [0, 64)                 Meta, written by the parse kernel
//   [64, 64 + raw_pad)      inflated scanlines (raw_pad = raw_size rounded to 16,
//                           plus 256 bytes that the tiled unfilter's aligned
//                           16-byte reads may run over the last row)
//   [64 + raw_pad, ...)     the zlib stream: the data of the IDAT run gathered
//                           into one contiguous buffer, then 16 zero bytes
//                           (src_len + 16 rounded to 16 bytes are reserved)
struct Meta {
  uint64_t idat_pos;    // file offset of the first IDAT chunk (its length field)
  uint64_t plte_pos;    // file offset of the PLTE data (0: none)
  uint64_t trns_pos;    // file offset of the tRNS data (0: none)
  uint32_t plte_len, trns_len;
  uint64_t z_len;       // gathered zlib stream bytes
  uint64_t bad_zoff;    // stream offset where the first IDAT with a bad CRC
                        // starts (~0: none); an error once the stream reaches it
  int32_t status;
  int32_t depth, ctype, interlace;
};
static_assert(sizeof(Meta) == kMetaBytes, "Meta is one 64-byte record");
static_assert(kMetaBytes % 16 == 0, "the scanlines start 16-byte aligned");

__host__ __device__ inline uint64_t align16(uint64_t v) { return (v + 15) & ~uint64_t(15); }
constexpr uint64_t kRawSlack = 256;
__host__ __device__ inline uint64_t zstream_off(uint64_t raw) {
  return kMetaBytes + align16(raw) + kRawSlack;
}
__host__ __device__ inline uint64_t scratch_size(uint64_t raw, uint64_t src_len) {
  return zstream_off(raw) + align16(src_len + 16);
}

__host__ __device__ inline uint32_t be32(const uint8_t *p) {
  return (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | uint32_t(p[3]);
}

__host__ __device__ inline int channels_of(int ct) {
  return ct == 0 ? 1 : ct == 2 ? 3 : ct == 3 ? 1 : ct == 4 ? 2 : ct == 6 ? 4 : 0;
}

// Valid (colour type, bit depth) pairs of the PNG specification.
__host__ __device__ inline bool depth_ok(int ct, int d) {
  switch (ct) {
    case 0: return d == 1 || d == 2 || d == 4 || d == 8 || d == 16;
    case 3: return d == 1 || d == 2 || d == 4 || d == 8;
    case 2: case 4: case 6: return d == 8 || d == 16;
    default: return false;
  }
}

// Adam7 pass geometry (x0, y0, dx, dy), or the single pass of a
// non-interlaced image.
__host__ __device__ inline void pass_geom(int interlace, int p, int &x0, int &y0, int &dx, int &dy) {
  if (!interlace) { x0 = 0; y0 = 0; dx = 1; dy = 1; return; }
  const int8_t t[7][4] = {{0, 0, 8, 8}, {4, 0, 8, 8}, {0, 4, 4, 8}, {2, 0, 4, 4},
                          {0, 2, 2, 4}, {1, 0, 2, 2}, {0, 1, 1, 2}};
  x0 = t[p][0]; y0 = t[p][1]; dx = t[p][2]; dy = t[p][3];
}

__host__ __device__ inline uint64_t row_bytes(uint64_t w, int ch, int depth) {
  return (w * ch * depth + 7) / 8;
}

// Bytes of the inflated stream: every pass's rows, each with its filter byte.
__host__ __device__ inline uint64_t raw_size(uint64_t w, uint64_t h, int ct, int depth, int il) {
  const int ch = channels_of(ct);
  uint64_t total = 0;
  for (int p = 0; p < (il ? 7 : 1); ++p) {
    int x0, y0, dx, dy;
    pass_geom(il, p, x0, y0, dx, dy);
    const uint64_t pw = w > (uint64_t)x0 ? (w - x0 + dx - 1) / dx : 0;
    const uint64_t ph = h > (uint64_t)y0 ? (h - y0 + dy - 1) / dy : 0;
    if (pw && ph) total += ph * (1 + row_bytes(pw, ch, depth));
  }
  return total;
}

// ---- CRC-32 arithmetic (reflected bit order: bit 31 holds x^0) ----
// a * b mod P over GF(2).
__host__ __device__ inline uint32_t gf_mul(uint32_t a, uint32_t b) {
  uint32_t p = 0;
  for (int i = 0; i < 32; ++i) {
    if (a & 0x80000000u) p ^= b;
    a <<= 1;
    b = (b & 1u) ? (b >> 1) ^ kCrcPoly : b >> 1;
  }
  return p;
}

// x^(8n) mod P: the operator that advances a CRC register over n zero bytes.
__host__ __device__ inline uint32_t x8n(uint64_t n) {
  uint32_t r = 0x80000000u, base = 0x00800000u;  // x^0, x^8
  while (n) {
    if (n & 1) r = gf_mul(r, base);
    base = gf_mul(base, base);
    n >>= 1;
  }
  return r;
}


constexpr uint32_t kFull = 0xFFFFFFFFu;
constexpr uint32_t kIHDR = 0x49484452u, kPLTE = 0x504C5445u, kIDAT = 0x49444154u,
                   kTRNS = 0x74524E53u;

// ---- parse kernel ----
constexpr int kParseWarps = 4;

struct CrcTables {
  uint32_t t[4][256];  // slice-by-4 tables
  uint32_t m[6];       // x^(8*256*2^l) mod P for l = 0..4, x^(8*8192) mod P
};

__device__ void build_crc_tables(CrcTables &ct) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    uint32_t c = i;
    for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kCrcPoly : c >> 1;
    ct.t[0][i] = c;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    uint32_t c = ct.t[0][i];
    for (int k = 1; k < 4; ++k) {
      c = ct.t[0][c & 0xFFu] ^ (c >> 8);
      ct.t[k][i] = c;
    }
  }
  if (threadIdx.x < 6) ct.m[threadIdx.x] = x8n(threadIdx.x < 5 ? (256ull << threadIdx.x) : 8192ull);
  __syncthreads();
}

// CRC register r advanced over n bytes at p (no pre/post conditioning).
__device__ uint32_t crc_run(uint32_t r, const uint8_t *p, uint32_t n, const CrcTables &ct) {
  uint32_t i = 0;
  for (; i + 4 <= n; i += 4) {
    r ^= uint32_t(p[i]) | (uint32_t(p[i + 1]) << 8) | (uint32_t(p[i + 2]) << 16) |
         (uint32_t(p[i + 3]) << 24);
    r = ct.t[3][r & 0xFFu] ^ ct.t[2][(r >> 8) & 0xFFu] ^ ct.t[1][(r >> 16) & 0xFFu] ^
        ct.t[0][r >> 24];
  }
  for (; i < n; ++i) r = ct.t[0][(r ^ p[i]) & 0xFFu] ^ (r >> 8);
  return r;
}

// CRC-32 of n bytes at p by the whole warp: rounds of up to 32 pieces of 256
// bytes (right-aligned on the lanes, so every right subtree of the combine
// tree is full), a 5-level shuffle tree joins them, lane 0's result shifts
// the running register; the last n % 256 bytes continue it directly. When
// `gather` is set, bytes [data_from, n) are also copied to gather (offset 0 =
// byte data_from). Every lane returns the same value.
__device__ uint32_t warp_crc(const uint8_t *p, uint64_t n, const CrcTables &ct, int lane,
                             uint8_t *gather = nullptr, uint64_t data_from = 0) {
  uint32_t S = kFull;
  const uint64_t nfull = n / 256;
  for (uint64_t base = 0; base < nfull; base += 32) {
    const int k = (int)(nfull - base < 32 ? nfull - base : 32);
    const int seg = lane - (32 - k);
    uint32_t r = 0;
    if (seg >= 0) r = crc_run(0, p + (base + seg) * 256, 256, ct);
#pragma unroll
    for (int l = 0; l < 5; ++l) {
      const uint32_t right = __shfl_down_sync(kFull, r, 1 << l);
      if ((lane & ((2 << l) - 1)) == 0) r = gf_mul(r, ct.m[l]) ^ right;
    }
    r = __shfl_sync(kFull, r, 0);
    uint32_t op = ct.m[5];
    if (k < 32) {
      op = 0x80000000u;
      for (int l = 0; l < 5; ++l)
        if (k & (1 << l)) op = gf_mul(op, ct.m[l]);
    }
    S = gf_mul(S, op) ^ r;
  }
  S = crc_run(S, p + nfull * 256, (uint32_t)(n - nfull * 256), ct);
  if (gather)
    for (uint64_t i = data_from + lane; i < n; i += 32) gather[i - data_from] = p[i];
  return S ^ kFull;
}

// Everything before the image data, as Wuffs' PNG decoder checks it
// (decode_ihdr, decode_other_chunk, decode_plte, decode_trns in
// third_party/wuffs/wuffs-v0.4.c), then the CRCs and the gather of the IDAT
// run. Warp-uniform: every lane walks the same chunks.
__device__ int parse_one(const uint8_t *f, uint64_t L, const tocr_png_job &job, Meta &m,
                         uint8_t *base, const CrcTables &ct, int lane) {
  const uint8_t sig[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
  if (L < 33) return kBadHeader;
  for (int i = 0; i < 8; ++i)
    if (f[i] != sig[i]) return kBadHeader;
  if (be32(f + 8) != 13 || be32(f + 12) != kIHDR) return kBadHeader;
  const uint32_t w = be32(f + 16), h = be32(f + 20);
  if (w == 0 || h == 0 || w > 0x7FFFFFFFu || h > 0x7FFFFFFFu) return kBadHeader;
  if (w > 16777215u || h > 16777215u) return kUnsupported;
  const int depth = f[24], ctype = f[25], il = f[28];
  if (!depth_ok(ctype, depth) || f[26] != 0 || f[27] != 0 || il > 1) return kBadHeader;
  if (warp_crc(f + 12, 17, ct, lane) != be32(f + 29)) return kBadChecksum;
  if ((int64_t)w != job.width || (int64_t)h != job.height) return kSizeMismatch;
  m.depth = depth;
  m.ctype = ctype;
  m.interlace = il;
  uint8_t *zbuf = base + zstream_off(raw_size(w, h, ctype, depth, il));
  uint64_t pos = 33;
  bool plte = false, trns = false;
  for (;;) {  // pos grows by >= 12 per chunk
    if (pos + 8 > L) return kBadChunk;
    const uint32_t clen = be32(f + pos), type = be32(f + pos + 4);
    if (clen > 0x7FFFFFFFu || pos + 12 + (uint64_t)clen > L) return kBadChunk;
    if (type == kIDAT) break;
    const bool critical = ((type >> 24) & 0x20u) == 0;
    if (type == kPLTE) {
      if (ctype == 0 || ctype == 4 || plte || trns) return kBadChunk;
      if (clen % 3 != 0 || clen > 768) return kBadChunk;
      if (warp_crc(f + pos + 4, 4 + (uint64_t)clen, ct, lane) != be32(f + pos + 8 + clen))
        return kBadChecksum;
      plte = true;
      m.plte_pos = pos + 8;
      m.plte_len = clen;
    } else if (type == kTRNS) {
      if (trns) return kBadChunk;
      if (ctype == 0 && clen != 2) return kBadChunk;
      if (ctype == 2 && clen != 6) return kBadChunk;
      if (ctype == 3 && (!plte || clen > 256)) return kBadChunk;
      trns = true;
      if (ctype == 0 || ctype == 2 || ctype == 3) {
        m.trns_pos = pos + 8;
        m.trns_len = clen;
      }
    } else if (critical) {
      return kBadChunk;  // IHDR again, IEND before the data, or unknown
    }
    pos += 12 + (uint64_t)clen;
  }
  if (ctype == 3 && !plte) return kMissingPalette;
  m.idat_pos = pos;
  // The IDAT run: CRC of each chunk (type + data) and its data gathered.
  uint64_t z = 0;
  while (pos + 8 <= L && be32(f + pos + 4) == kIDAT) {
    const uint32_t clen = be32(f + pos);
    if (clen > 0x7FFFFFFFu || pos + 12 + (uint64_t)clen > L) break;  // truncated: the stream ends here
    const uint32_t crc = warp_crc(f + pos + 4, 4 + (uint64_t)clen, ct, lane, zbuf + z, 4);
    if (crc != be32(f + pos + 8 + clen) && m.bad_zoff == ~0ull) m.bad_zoff = z;
    z += clen;
    pos += 12 + (uint64_t)clen;
  }
  m.z_len = z;
  for (int i = lane; i < 16; i += 32) zbuf[z + i] = 0;
  return kOk;
}

__global__ void __launch_bounds__(kParseWarps * 32)
png_parse_kernel(const uint8_t *__restrict__ src, const tocr_png_job *__restrict__ jobs, int n,
                 uint8_t *__restrict__ scratch) {
  __shared__ CrcTables ct;
  build_crc_tables(ct);
  const int lane = threadIdx.x & 31;
  const int img = blockIdx.x * kParseWarps + (threadIdx.x >> 5);
  if (img >= n) return;
  const tocr_png_job job = jobs[img];
  Meta m;
  memset(&m, 0, sizeof m);
  m.bad_zoff = ~0ull;
  uint8_t *base = scratch + job.scratch_off;
  m.status = parse_one(src + job.src_off, job.src_len, job, m, base, ct, lane);
  if (lane == 0) *reinterpret_cast<Meta *>(base) = m;
}

// ---- inflate kernel ----
// RFC 1951 section 3.2.5: base values and extra bits of the length symbols
// 257..285 and the distance symbols 0..29, and the order in which the
// code-length code's lengths are sent (3.2.7).
__constant__ uint16_t kLenBase[29] = {3,  4,  5,  6,  7,  8,  9,  10, 11,  13,  15,  17,  19,  23, 27,
                                      31, 35, 43, 51, 59, 67, 83, 99, 115, 131, 163, 195, 227, 258};
__constant__ uint8_t kLenExtra[29] = {0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2,
                                      2, 3, 3, 3, 3, 4, 4, 4, 4, 5, 5, 5, 5, 0};
__constant__ uint16_t kDistBase[30] = {1,    2,    3,    4,    5,    7,     9,     13,    17,  25,
                                       33,   49,   65,   97,   129,  193,   257,   385,   513, 769,
                                       1025, 1537, 2049, 3073, 4097, 6145, 8193, 12289, 16385, 24577};
__constant__ uint8_t kDistExtra[30] = {0, 0, 0, 0, 1, 1, 2, 2,  3,  3,  4,  4,  5,  5,  6,
                                       6, 7, 7, 8, 8, 9, 9, 10, 10, 11, 11, 12, 12, 13, 13};
__constant__ uint8_t kClOrder[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};

// Two warps per image: a decoder warp (lane 0 walks the bit stream; the
// whole warp builds the Huffman tables) fills a batch of tokens while the
// copier warp applies the previous batch to the 32 KB window, flushes it to
// the scanline buffer and folds it into the Adler-32. The two meet at a
// named barrier after every batch (double-buffered batches), so decoding and
// copying overlap.
constexpr int kInfImgs = 1;                 // images per CTA: small batches spread over the SMs
constexpr uint32_t kWin = 32768, kWinMask = kWin - 1;
constexpr int kFastBits = 10;
constexpr int kPairBits = 11;               // two-literal table: both codes within 11 bits
constexpr int kMaxTok = 128;
constexpr int kMaxLit = 1024;
constexpr uint32_t kFlush = 4096;
constexpr uint32_t kAdlerMod = 65521;
constexpr uint16_t kStoredTok = 0xFFFF;     // token dist of a stored-block copy from the stream

// Canonical Huffman code: a 10-bit first-level table and, for the longer
// codes, the counts per length with the symbols sorted by (length, value).
struct Huff {
  uint16_t fast[1 << kFastBits];  // symbol | length << 9; 0: walk the canonical code
  uint16_t count[16];
  uint16_t offs[16];
  uint16_t first[16];             // first code of each length
  uint16_t sorted[288];
};

// One batch: the literals in lit[] and the tokens, each a run of litc[k]
// literals (taken from lit[] in order) followed by either an LZ77 match
// (dist 1..32768, len bytes) or, for dist == kStoredTok, len bytes copied
// from the stream at src; the literals after the last token close the batch.
struct Batch {
  uint16_t len[kMaxTok];
  uint16_t dist[kMaxTok];
  uint16_t litc[kMaxTok];
  uint32_t src[kMaxTok];
  uint8_t lit[kMaxLit];
  int ntok, nlit;
  int last;    // the decoder has nothing after this batch
  int pad;
};

struct alignas(16) InflateImg {  // 16-byte aligned: the window is read as uint4
  uint8_t win[kWin];
  Huff lit, dist;                 // `dist` also holds the code-length code
  uint32_t pair[1 << kPairBits];  // literal pairs of the current literal/length code
  Batch batch[2];
  uint16_t run[16];
  uint8_t lens[320];
  uint8_t cl[20];
  int dec_status;                 // decoder's verdict (kOk until an error)
  uint32_t adler_want;            // the stream's Adler-32
};
static_assert(sizeof(InflateImg) % 16 == 0, "per-image regions stay 16-byte aligned");
static_assert(sizeof(InflateImg) * kInfImgs <= 227 * 1024, "shared memory per CTA");

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Builds `h` from nsym code lengths (warp-wide). Over-subscribed codes, an
// all-zero set and incomplete codes are errors, except that a distance code
// may be a single code of length 1 (the rules of Wuffs' init_huff).
__device__ int build_huff(Huff &h, const uint8_t *lens, int nsym, bool is_dist, uint16_t *run,
                          int lane) {
  for (int i = lane; i < (1 << kFastBits); i += 32) h.fast[i] = 0;
  if (lane < 16) run[lane] = 0;
  __syncwarp();
  const unsigned lt = (1u << lane) - 1u;
  for (int b = 0; b < nsym; b += 32) {
    const int s = b + lane;
    const int l = s < nsym ? lens[s] : 0;
    const unsigned mask = __match_any_sync(kFull, l);
    if (l && lane == __ffs(mask) - 1) run[l] += __popc(mask);
    __syncwarp();
  }
  int st = kOk;
  if (lane == 0) {
    int total = 0, left = 1;
    h.count[0] = 0;
    for (int l = 1; l < 16; ++l) {
      h.count[l] = run[l];
      total += run[l];
      left = (left << 1) - run[l];
      if (left < 0) st = kBadDeflate;
    }
    if (total == 0) st = kBadDeflate;
    if (st == kOk && left != 0 && !(is_dist && total == 1 && h.count[1] == 1)) st = kBadDeflate;
    int off = 0, code = 0;
    for (int l = 1; l < 16; ++l) {
      code = (code + h.count[l - 1]) << 1;
      h.first[l] = (uint16_t)code;
      h.offs[l] = (uint16_t)off;
      off += h.count[l];
      run[l] = 0;
    }
  }
  st = __shfl_sync(kFull, st, 0);
  __syncwarp();
  if (st != kOk) return st;
  for (int b = 0; b < nsym; b += 32) {
    const int s = b + lane;
    const int l = s < nsym ? lens[s] : 0;
    const unsigned mask = __match_any_sync(kFull, l);
    const int rank = l ? run[l] + __popc(mask & lt) : 0;
    __syncwarp();
    if (l && lane == __ffs(mask) - 1) run[l] += __popc(mask);
    if (l) {
      h.sorted[h.offs[l] + rank] = (uint16_t)s;
      if (l <= kFastBits) {
        const uint32_t code = h.first[l] + rank;
        const uint16_t e = (uint16_t)(s | (l << 9));
        for (uint32_t j = __brev(code) >> (32 - l); j < (1u << kFastBits); j += 1u << l) h.fast[j] = e;
      }
    }
    __syncwarp();
  }
  return kOk;
}

// The canonical walk for codes the first-level table does not hold (longer
// than kFastBits, or none), kept out of line so the hot loops stay small.
// Returns symbol | bits << 16, or -1.
__device__ __noinline__ int decode_sym_slow(const Huff &h, uint64_t buf) {
  int code = 0, first = 0, index = 0;
#pragma unroll 1
  for (int len = 1; len < 16; ++len) {
    code |= (int)(buf & 1u);
    buf >>= 1;
    const int c = h.count[len];
    if (code - c < first) return h.sorted[index + (code - first)] | (len << 16);
    index += c;
    first = (first + c) << 1;
    code <<= 1;
  }
  return -1;
}

// One symbol from the bit buffer (at least 15 valid bits); -1 for a code
// the table does not hold.
__device__ __forceinline__ int decode_sym(const Huff &h, uint64_t &buf, int &cnt) {
  const uint32_t e = h.fast[buf & ((1u << kFastBits) - 1)];
  int l = (int)(e >> 9), sym = (int)(e & 511u);
  if (!l) {
    const int r = decode_sym_slow(h, buf);
    if (r < 0) return -1;
    l = r >> 16;
    sym = r & 0xFFFF;
  }
  buf >>= l;
  cnt -= l;
  return sym;
}

// Brings the line at p into L1 ahead of its use (no value, no fault on a
// valid address; callers stay inside the stream).
__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Lane 0's bit reader over the gathered zlib stream (16-byte aligned, zero
// bytes readable past its end). Whole 32-bit words are appended, the next
// one loaded a refill ahead and its line 256 bytes ahead prefetched into L1,
// so that neither latency sits on the decoding chain.
// Bytes appended from past the stream's end are counted in `over`.
struct BitReader {
  const uint32_t *zw;
  uint64_t zlen, wi, buf;  // wi: words appended so far
  int cnt;
  uint32_t nextw;

  __device__ void init(const uint8_t *z, uint64_t len) {
    zw = reinterpret_cast<const uint32_t *>(z);
    zlen = len;
    wi = 0;
    buf = 0;
    cnt = 0;
    nextw = zw[0];
  }
  // Bytes appended from past the stream's end (they read as zeros).
  __device__ __forceinline__ uint32_t over() const {
    return wi * 4 > zlen ? (uint32_t)(wi * 4 - zlen) : 0u;
  }
  // The stream is read more than 8 bytes past its end: the data is truncated.
  __device__ __forceinline__ bool runaway() const { return wi * 4 > zlen + 8; }
  // Leaves at least 32 bits in the buffer. The word after the last one
  // appended is always loaded (at most 16 bytes past the end, which the
  // layout reserves as zeros) unless the reader has run away.
  __device__ __forceinline__ void refill() {
    if (cnt < 32) {
      buf |= uint64_t(nextw) << cnt;
      cnt += 32;
      ++wi;
      if (!runaway()) {
        nextw = zw[wi];
        if ((wi + 64) * 4 < zlen) prefetch_l1(zw + wi + 64);
      }
    }
  }
  __device__ __forceinline__ uint32_t bits(int n) {  // n <= 32, cnt >= n
    const uint32_t v = (uint32_t)(buf & ((1ull << n) - 1ull));
    buf >>= n;
    cnt -= n;
    return v;
  }
  // A byte from past the stream's end has been consumed.
  __device__ __forceinline__ bool overrun() const { return cnt < (int)over() * 8; }
  // Stream offset of the next unconsumed byte (at a byte boundary).
  __device__ __forceinline__ uint64_t pos() const { return wi * 4 - (uint64_t)(cnt >> 3); }
  // Continue at byte offset p (p <= zlen).
  __device__ void seek(uint64_t p) {
    wi = p >> 2;
    buf = 0;
    cnt = 0;
    nextw = zw[wi];
    refill();
    bits((int)(p & 3) * 8);
  }
};

__device__ __forceinline__ uint32_t mod_adler(uint64_t v) { return (uint32_t)(v % kAdlerMod); }

// Copier: window bytes [from, from + n) to raw (from a multiple of kFlush,
// n <= kFlush), folded into the Adler-32 (a, b).
__device__ void flush_block(const uint8_t *win, uint8_t *raw, uint64_t from, uint32_t n,
                            uint32_t &a, uint32_t &b, int lane) {
  const uint8_t *w = win + (from & kWinMask);
  uint32_t s = 0;
  uint64_t t = 0;
  if (n == kFlush) {
    uint4 *dst = reinterpret_cast<uint4 *>(raw + from);
    const uint4 *srcv = reinterpret_cast<const uint4 *>(w);
    for (int i = lane; i < (int)(kFlush / 16); i += 32) {
      const uint4 v = srcv[i];
      dst[i] = v;
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t off = i * 16 + k * 4;
        const uint32_t sum = __dp4a(words[k], 0x01010101u, 0u);
        const uint32_t wsum = __dp4a(words[k], 0x03020100u, 0u);
        s += sum;
        t += (uint64_t)(n - off) * sum - wsum;
      }
    }
  } else {
    for (uint32_t i = lane; i < n; i += 32) {
      const uint8_t v = w[i];
      raw[from + i] = v;
      s += v;
      t += (uint64_t)(n - i) * v;
    }
  }
  uint32_t tm = mod_adler(t);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(kFull, s, o);
    tm += __shfl_xor_sync(kFull, tm, o);
  }
  const uint32_t a0 = a;
  a = mod_adler((uint64_t)a0 + s);
  b = mod_adler((uint64_t)b + (uint64_t)n * a0 + tm);
}

__device__ __forceinline__ void flush_ready(const uint8_t *win, uint8_t *raw, uint64_t out,
                                            uint64_t &flushed, uint32_t &a, uint32_t &b, bool last,
                                            int lane) {
  while (out - flushed >= kFlush) {
    flush_block(win, raw, flushed, kFlush, a, b, lane);
    flushed += kFlush;
  }
  if (last && out > flushed) {
    flush_block(win, raw, flushed, (uint32_t)(out - flushed), a, b, lane);
    flushed = out;
  }
}

// Copier warp: applies one batch to the window in token order. Token
// fields are read once per 32 tokens and their output and literal offsets
// scanned across the lanes; a match loads all its source bytes before
// storing (its sources lie before its first byte), so it costs one
// shared-memory round trip. The window is flushed whenever 4 KB are
// complete, which keeps the unflushed part under 4 KB + 770 bytes and every
// match source inside the window.
__device__ __forceinline__ void copy_lits(InflateImg &S, const Batch &B, uint64_t at, int from,
                                          uint32_t n, int lane) {
  for (uint32_t i = lane; i < n; i += 32) S.win[(at + i) & kWinMask] = B.lit[from + i];
}

__device__ void run_batch(InflateImg &S, const Batch &B, const uint8_t *z, uint8_t *raw,
                          uint64_t &out, uint64_t &flushed, uint32_t &ad_a, uint32_t &ad_b,
                          int lane) {
  const int ntok = B.ntok;
  int litpos = 0;
  for (int base = 0; base < ntok; base += 32) {
    const int k = base + lane;
    const uint32_t myl = k < ntok ? B.len[k] : 0u;
    const uint32_t myd = k < ntok ? B.dist[k] : 0u;
    const uint32_t myc = k < ntok ? B.litc[k] : 0u;
    uint32_t o = myl + myc, lo = myc;
#pragma unroll
    for (int sh = 1; sh < 32; sh <<= 1) {
      const uint32_t x = __shfl_up_sync(kFull, o, sh), y = __shfl_up_sync(kFull, lo, sh);
      if (lane >= sh) {
        o += x;
        lo += y;
      }
    }
    const uint32_t tot = __shfl_sync(kFull, o, 31), ltot = __shfl_sync(kFull, lo, 31);
    o -= myl + myc;
    lo -= myc;
    const int nt = ntok - base < 32 ? ntok - base : 32;
    for (int t = 0; t < nt; ++t) {
      const uint32_t len = __shfl_sync(kFull, myl, t), d = __shfl_sync(kFull, myd, t);
      const uint32_t nl = __shfl_sync(kFull, myc, t);
      uint64_t at = out + __shfl_sync(kFull, o, t);
      if (nl) {
        copy_lits(S, B, at, litpos + (int)__shfl_sync(kFull, lo, t), nl, lane);
        at += nl;
        __syncwarp();
      }
      if (d != kStoredTok) {
        uint8_t v[9];
        const uint32_t step = d > 32 ? 32u : 32u % d;
        uint32_t si = d > 32 ? (uint32_t)lane : (uint32_t)lane % d;
        const uint64_t from = at - d;
        const int nu = (int)((len + 31) >> 5);
#pragma unroll
        for (int u = 0; u < 9; ++u) {
          if (u < nu) {
            if (lane + 32u * u < len) v[u] = S.win[(from + si) & kWinMask];
            si += step;
            if (si >= d) si -= d;
          }
        }
#pragma unroll
        for (int u = 0; u < 9; ++u)
          if (u < nu && lane + 32u * u < len) S.win[(at + lane + 32u * u) & kWinMask] = v[u];
      } else {
        const uint64_t src = B.src[base + t];
        for (uint32_t done = 0; done < len;) {
          const uint32_t chunk = len - done < 8192u ? len - done : 8192u;
          for (uint32_t i = lane; i < chunk; i += 32)
            S.win[(at + done + i) & kWinMask] = z[src + done + i];
          done += chunk;
          __syncwarp();
          flush_ready(S.win, raw, at + done, flushed, ad_a, ad_b, false, lane);
        }
      }
      __syncwarp();
      if (at + len - flushed >= kFlush) {
        flush_ready(S.win, raw, at + len, flushed, ad_a, ad_b, false, lane);
        __syncwarp();
      }
    }
    out += tot;
    litpos += (int)ltot;
  }
  const uint32_t tail = (uint32_t)(B.nlit - litpos);
  if (tail) {
    copy_lits(S, B, out, litpos, tail, lane);
    out += tail;
    __syncwarp();
    flush_ready(S.win, raw, out, flushed, ad_a, ad_b, false, lane);
    __syncwarp();
  }
}

// The two-literal table of the current literal/length code: entry i holds
// the first code of the bits i (least significant first) and the code after
// it when both are literals whose lengths add up to at most kPairBits, as
// sym1 | sym2 << 8 | (len1 + len2) << 16 | 2 << 24; 0 otherwise. A literal
// run (5 bits per literal on document pages) then takes one lookup per two
// literals on the decoder's dependent chain.
__device__ void build_pairs(InflateImg &S, int lane) {
  __syncwarp();
  for (int i = lane; i < (1 << kPairBits); i += 32) {
    uint32_t v = 0;
    const uint32_t e1 = S.lit.fast[i & ((1 << kFastBits) - 1)];
    const uint32_t l1 = e1 >> 9, s1 = e1 & 511u;
    if (l1 != 0 && s1 < 256 && l1 < (uint32_t)kPairBits) {
      const uint32_t e2 = S.lit.fast[((uint32_t)i >> l1) & ((1u << kFastBits) - 1)];
      const uint32_t l2 = e2 >> 9, s2 = e2 & 511u;
      if (l2 != 0 && s2 < 256 && l1 + l2 <= (uint32_t)kPairBits)
        v = s1 | s2 << 8 | (l1 + l2) << 16 | 2u << 24;
    }
    S.pair[i] = v;
  }
  __syncwarp();
}

__device__ void build_fixed(InflateImg &S, int lane) {
  for (int i = lane; i < 320; i += 32)
    S.lens[i] = i < 144 ? 8 : i < 256 ? 9 : i < 280 ? 7 : i < 288 ? 8 : 5;
  __syncwarp();
  build_huff(S.lit, S.lens, 288, false, S.run, lane);
  build_huff(S.dist, S.lens + 288, 32, true, S.run, lane);
  build_pairs(S, lane);
}

// The dynamic block header (RFC 1951 3.2.7) with Wuffs' checks: at most 286
// literal/length and 30 distance codes, no repeat before the first length,
// no run past the end, a non-zero length for the end-of-block code.
__device__ int read_dynamic(InflateImg &S, BitReader &br, int lane) {
  int st = kOk, hlit = 0, hdist = 0;
  if (lane == 0) {
    br.refill();
    hlit = (int)br.bits(5) + 257;
    hdist = (int)br.bits(5) + 1;
    const int hclen = (int)br.bits(4) + 4;
    if (hlit > 286 || hdist > 30) st = kBadDeflate;
    for (int i = 0; i < 19; ++i) S.cl[i] = 0;
    for (int i = 0; i < hclen; ++i) {
      br.refill();
      S.cl[kClOrder[i]] = (uint8_t)br.bits(3);
    }
    if (br.runaway()) st = kBadChunk;
  }
  st = __shfl_sync(kFull, st, 0);
  hlit = __shfl_sync(kFull, hlit, 0);
  hdist = __shfl_sync(kFull, hdist, 0);
  __syncwarp();
  if (st != kOk) return st;
  st = build_huff(S.dist, S.cl, 19, false, S.run, lane);
  if (st != kOk) return st;
  if (lane == 0) {
    const int total = hlit + hdist;
    int i = 0;
    while (i < total && st == kOk) {
      br.refill();
      if (br.runaway()) { st = kBadChunk; break; }
      const int sym = decode_sym(S.dist, br.buf, br.cnt);
      if (sym < 0) { st = kBadDeflate; break; }
      if (sym < 16) { S.lens[i++] = (uint8_t)sym; continue; }
      int rep;
      uint8_t val = 0;
      if (sym == 16) {
        if (i == 0) { st = kBadDeflate; break; }
        val = S.lens[i - 1];
        rep = 3 + (int)br.bits(2);
      } else if (sym == 17) {
        rep = 3 + (int)br.bits(3);
      } else {
        rep = 11 + (int)br.bits(7);
      }
      if (i + rep > total) { st = kBadDeflate; break; }
      while (rep--) S.lens[i++] = val;
    }
    if (st == kOk && S.lens[256] == 0) st = kBadDeflate;
  }
  st = __shfl_sync(kFull, st, 0);
  __syncwarp();
  if (st != kOk) return st;
  st = build_huff(S.lit, S.lens, hlit, false, S.run, lane);
  if (st != kOk) return st;
  build_pairs(S, lane);
  return build_huff(S.dist, S.lens + hlit, hdist, true, S.run, lane);
}

// Decoder state carried from batch to batch (block state is warp-uniform;
// the bit reader lives in lane 0).
struct DecState {
  BitReader br;
  uint64_t produced;  // bytes the tokens so far produce
  int in_block;       // inside a Huffman-coded block
  int final_seen;     // the last block header had BFINAL set
  int fixed_ready;    // S.lit / S.dist hold the fixed code
};

// End of the stream, after the last block: the Adler-32 from the next byte
// boundary, the scanline count, the CRC of every IDAT the stream used, and
// no bytes after the stream inside its last IDAT (Wuffs reads no further).
__device__ int finish_stream(InflateImg &S, DecState &ds, const Meta &m, const uint8_t *f,
                             uint64_t L, uint64_t raw_total, uint64_t produced) {
  BitReader &br = ds.br;
  br.bits(br.cnt & 7);
  br.refill();
  uint32_t want = 0;
  for (int i = 0; i < 4; ++i) want = (want << 8) | br.bits(8);
  S.adler_want = want;
  if (br.overrun()) return kBadChunk;
  if (produced < raw_total) return kNotEnoughData;
  const uint64_t end = br.pos();
  if (m.bad_zoff != ~0ull && end > m.bad_zoff) return kBadChecksum;
  uint64_t pos = m.idat_pos, cum = 0;
  while (pos + 12 <= L) {
    const uint64_t clen = be32(f + pos);
    if (end <= cum + clen) return end < cum + clen ? kTooMuchData : kOk;
    cum += clen;
    pos += 12 + clen;
  }
  return kOk;
}

// Decoder warp: fills B with tokens (reading block headers and building
// tables on the way) until B is full or the stream has ended; sets B.last
// and S.dec_status at the end or on the first error. The output count is
// checked against the scanline size once per batch: a batch that would
// pass it is dropped whole and ends the stream with kTooMuchData.
__device__ void fill_batch(InflateImg &S, Batch &B, DecState &ds, const Meta &m, const uint8_t *f,
                           uint64_t L, uint64_t raw_total, int lane) {
  int ntok = 0, nlit = 0, st = kOk, last = 0;
  uint32_t lit_mark = 0;  // literals already attached to a token
  uint64_t msum = 0;      // bytes of this batch's matches and stored copies
  for (;;) {
    if (!ds.in_block) {
      if (ds.final_seen) {
        if (lane == 0) st = finish_stream(S, ds, m, f, L, raw_total, ds.produced + nlit + msum);
        st = __shfl_sync(kFull, st, 0);
        last = 1;
        break;
      }
      if (ntok > kMaxTok - 1 || nlit > kMaxLit - 8) break;  // room for a stored block
      int fin = 0, type = 0;
      if (lane == 0) {
        BitReader &br = ds.br;
        br.refill();
        fin = (int)br.bits(1);
        type = (int)br.bits(2);
        if (br.runaway()) st = kBadChunk;
        else if (type == 3) st = kBadDeflate;
        else if (type == 0) {
          // Stored: LEN, NLEN, then LEN bytes: those still in the bit buffer
          // as literals, the rest as a copy straight from the stream.
          br.bits(br.cnt & 7);
          br.refill();
          const uint32_t len = br.bits(16), nlen = br.bits(16);
          if (len != (~nlen & 0xFFFFu)) st = kBadDeflate;
          else if (br.overrun()) st = kBadChunk;
          else {
            const uint32_t real = (uint32_t)(br.cnt >> 3) - br.over();
            const uint32_t k = len < real ? len : real;
            for (uint32_t i = 0; i < k; ++i) B.lit[nlit++] = (uint8_t)br.bits(8);
            if (len > k) {
              const uint64_t p = br.pos();
              if (p + (len - k) > br.zlen) {
                st = kBadChunk;
              } else {
                B.len[ntok] = (uint16_t)(len - k);
                B.dist[ntok] = kStoredTok;
                B.litc[ntok] = (uint16_t)(nlit - lit_mark);
                B.src[ntok] = (uint32_t)p;
                lit_mark = nlit;
                msum += len - k;
                ++ntok;
                br.seek(p + (len - k));
              }
            }
          }
        }
      }
      st = __shfl_sync(kFull, st, 0);
      fin = __shfl_sync(kFull, fin, 0);
      type = __shfl_sync(kFull, type, 0);
      ntok = __shfl_sync(kFull, ntok, 0);
      nlit = __shfl_sync(kFull, nlit, 0);
      if (st != kOk) { last = 1; break; }
      ds.final_seen = fin;
      if (type == 1) {
        if (!ds.fixed_ready) build_fixed(S, lane);
        ds.fixed_ready = 1;
        ds.in_block = 1;
      } else if (type == 2) {
        ds.fixed_ready = 0;
        st = read_dynamic(S, ds.br, lane);
        if (st != kOk) { last = 1; break; }
        ds.in_block = 1;
      }
      continue;
    }
    // Inside a Huffman block: lane 0 decodes until the batch is full or the
    // block ends. A literal costs a table lookup and one byte store.
    int eob = 0;
    if (lane == 0) {
      // The bit reader's state is copied into locals for the loop so that it
      // stays in registers; a literal costs one table lookup, two shifts and
      // one byte store.
      const uint32_t *zw = ds.br.zw;
      const uint64_t zlen = ds.br.zlen;
      uint64_t buf = ds.br.buf, wi = ds.br.wi;
      int cnt = ds.br.cnt;
      uint32_t nextw = ds.br.nextw;
      const uint64_t base = ds.produced;
      const uint16_t *lfast = S.lit.fast, *dfast = S.dist.fast;
      const uint32_t *pairs = S.pair;
      uint8_t *lit = B.lit;
      for (;;) {
        if (cnt < 32) {
          buf |= uint64_t(nextw) << cnt;
          cnt += 32;
          ++wi;
          if (wi * 4 > zlen + 8) { st = kBadChunk; break; }  // past the data: truncated
          nextw = zw[wi];
          if ((wi + 64) * 4 < zlen) prefetch_l1(zw + wi + 64);
        }
        const uint32_t pe = pairs[buf & ((1u << kPairBits) - 1)];
        if (pe != 0 && nlit + 2 <= kMaxLit) {  // two literals with short codes
          const int l2 = (int)((pe >> 16) & 255u);
          buf >>= l2;
          cnt -= l2;
          lit[nlit] = (uint8_t)pe;
          lit[nlit + 1] = (uint8_t)(pe >> 8);
          nlit += 2;
          if (nlit == kMaxLit) break;
          continue;
        }
        const uint32_t e = lfast[buf & ((1u << kFastBits) - 1)];
        int l = (int)(e >> 9), sym = (int)(e & 511u);
        if (l != 0 && sym < 256) {  // a literal with a short code
          buf >>= l;
          cnt -= l;
          lit[nlit++] = (uint8_t)sym;
          if (nlit == kMaxLit) break;
          continue;
        }
        if (!l) {
          const int r = decode_sym_slow(S.lit, buf);
          if (r < 0) { st = kBadDeflate; break; }
          l = r >> 16;
          sym = r & 0xFFFF;
        }
        buf >>= l;
        cnt -= l;
        if (sym < 256) {
          lit[nlit++] = (uint8_t)sym;
          if (nlit == kMaxLit) break;
          continue;
        }
        if (sym == 256) { eob = 1; break; }
        const int li = sym - 257;
        if (li >= 29) { st = kBadDeflate; break; }
        const int le = kLenExtra[li];
        const uint32_t len = kLenBase[li] + (uint32_t)(buf & ((1ull << le) - 1ull));
        buf >>= le;
        cnt -= le;
        if (cnt < 32) {
          buf |= uint64_t(nextw) << cnt;
          cnt += 32;
          ++wi;
          if (wi * 4 > zlen + 8) { st = kBadChunk; break; }
          nextw = zw[wi];
        }
        const uint32_t de = dfast[buf & ((1u << kFastBits) - 1)];
        int dl = (int)(de >> 9), dsym = (int)(de & 511u);
        if (!dl) {
          const int r = decode_sym_slow(S.dist, buf);
          if (r < 0) { st = kBadDeflate; break; }
          dl = r >> 16;
          dsym = r & 0xFFFF;
        }
        buf >>= dl;
        cnt -= dl;
        if (dsym >= 30) { st = kBadDeflate; break; }
        const int dx = kDistExtra[dsym];
        const uint32_t dist = kDistBase[dsym] + (uint32_t)(buf & ((1ull << dx) - 1ull));
        buf >>= dx;
        cnt -= dx;
        if (dist > base + nlit + msum) { st = kBadDeflate; break; }  // before the stream's first byte
        B.len[ntok] = (uint16_t)len;
        B.dist[ntok] = (uint16_t)dist;  // <= 32768
        B.litc[ntok] = (uint16_t)(nlit - lit_mark);
        lit_mark = nlit;
        msum += len;
        if (++ntok == kMaxTok) break;
      }
      ds.br.buf = buf;
      ds.br.cnt = cnt;
      ds.br.wi = wi;
      ds.br.nextw = nextw;
    }
    st = __shfl_sync(kFull, st, 0);
    eob = __shfl_sync(kFull, eob, 0);
    ntok = __shfl_sync(kFull, ntok, 0);
    nlit = __shfl_sync(kFull, nlit, 0);
    if (st != kOk) { last = 1; break; }
    if (eob) { ds.in_block = 0; continue; }
    break;  // the batch is full
  }
  if (lane == 0) {
    ds.produced += (uint64_t)nlit + msum;
    if (ds.produced > raw_total) {  // more scanline bytes than the IHDR allows
      ntok = 0;
      nlit = 0;
      st = kTooMuchData;
      last = 1;
    }
    B.ntok = ntok;
    B.nlit = nlit;
    B.last = last;
    if (last) S.dec_status = st;
  }
  ds.produced = __shfl_sync(kFull, ds.produced, 0);
  __syncwarp();
}

__global__ void __launch_bounds__(kInfImgs * 64)
png_inflate_kernel(const uint8_t *__restrict__ src, const tocr_png_job *__restrict__ jobs, int n,
                   uint8_t *__restrict__ scratch) {
  extern __shared__ __align__(16) uint8_t smem_inf[];
  const int slot = threadIdx.x >> 6, role = (threadIdx.x >> 5) & 1, lane = threadIdx.x & 31;
  const int img = blockIdx.x * kInfImgs + slot;
  if (img >= n) return;
  InflateImg &S = reinterpret_cast<InflateImg *>(smem_inf)[slot];
  const tocr_png_job job = jobs[img];
  uint8_t *base = scratch + job.scratch_off;
  const Meta m = *reinterpret_cast<const Meta *>(base);
  if (m.status != kOk) return;  // both warps leave before any barrier
  const uint64_t raw_total = raw_size(job.width, job.height, m.ctype, m.depth, m.interlace);
  const uint8_t *z = base + zstream_off(raw_total);
  uint8_t *raw = base + kMetaBytes;
  const int bar_id = 1 + slot;
  if (role == 0) {  // decoder
    DecState ds;
    ds.br.init(z, m.z_len);
    ds.produced = 0;
    ds.in_block = 0;
    ds.final_seen = 0;
    ds.fixed_ready = 0;
    int st = kOk;
    if (lane == 0) {
      BitReader &br = ds.br;
      br.refill();
      const uint32_t cmf = br.bits(8), flg = br.bits(8);
      if ((cmf & 15u) != 8u || (cmf >> 4) > 7u || ((cmf << 8) | flg) % 31u != 0u || (flg & 0x20u))
        st = kBadZlib;
      if (br.overrun()) st = kBadChunk;
      S.dec_status = kOk;
    }
    st = __shfl_sync(kFull, st, 0);
    bool last_seen = false;
    for (int iter = 0;; ++iter) {
      Batch &B = S.batch[iter & 1];
      if (!last_seen) {
        if (st != kOk) {  // the zlib header failed: an empty last batch
          if (lane == 0) {
            B.ntok = 0;
            B.last = 1;
            S.dec_status = st;
          }
          __syncwarp();
        } else {
          fill_batch(S, B, ds, m, src + job.src_off, job.src_len, raw_total, lane);
        }
      }
      named_bar(bar_id, 64);
      if (last_seen) break;
      last_seen = B.last != 0;
    }
  } else {  // copier
    uint64_t out = 0, flushed = 0;
    uint32_t ad_a = 1, ad_b = 0;
    bool last_seen = false;
    for (int iter = 0;; ++iter) {
      if (iter > 0) run_batch(S, S.batch[(iter - 1) & 1], z, raw, out, flushed, ad_a, ad_b, lane);
      named_bar(bar_id, 64);
      if (last_seen) break;
      last_seen = S.batch[iter & 1].last != 0;
    }
    flush_ready(S.win, raw, out, flushed, ad_a, ad_b, true, lane);
    int st = S.dec_status;
    if (st == kOk && S.adler_want != ((ad_b << 16) | ad_a)) st = kBadChecksum;
    if (lane == 0 && st != kOk) reinterpret_cast<Meta *>(base)->status = st;
  }
}

// ---- unfilter + colour conversion kernel ----

// Wuffs' 8-bit non-premultiplied to premultiplied step
// (wuffs_base__color_u32_argb_nonpremul__as__color_u32_argb_premul):
// widen colour and alpha to 16 bits by * 0x101, multiply, divide by 0xFFFF,
// narrow by >> 8.
__device__ __forceinline__ uint32_t premul(uint32_t c, uint32_t a) {
  return ((c * (a * 0x10201u)) / 0xFFFFu) >> 8;
}

__device__ __forceinline__ uint32_t paeth(uint32_t a, uint32_t b, uint32_t c) {
  const int p = (int)a + (int)b - (int)c;
  const int pa = abs(p - (int)a), pb = abs(p - (int)b), pc = abs(p - (int)c);
  return (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
}

struct Conv {
  int ctype, depth;
  uint32_t key[3];     // tRNS key samples (low `depth` bits), 1-8 bit grey / RGB
  bool has_key;
  const uint32_t *pal; // 256 premultiplied BGR entries (colour type 3)
};

__device__ __forceinline__ void put_bgr(uint8_t *px, uint32_t b, uint32_t g, uint32_t r) {
  px[0] = (uint8_t)b;
  px[1] = (uint8_t)g;
  px[2] = (uint8_t)r;
}

// Writes the pixel(s) of one reconstructed filter unit (BPP bytes in u,
// byte i at bits 8i). x is the unit's first pixel index within the pass row.
template <int BPP>
__device__ __forceinline__ void emit_unit(const Conv &cv, uint64_t u, int64_t x, int64_t pw,
                                          uint8_t *row_out, int x0, int dx) {
  const int ct = cv.ctype, d = cv.depth;
  if (d < 8) {  // BPP == 1: 8/d pixels, most significant bits first
    const uint32_t v8 = (uint32_t)(u & 0xFFu);
    const int per = 8 / d;
    const uint32_t mask = (1u << d) - 1u;
    for (int q = 0; q < per; ++q) {
      const int64_t xp = x * per + q;
      if (xp >= pw) break;
      const uint32_t v = (v8 >> (8 - d * (q + 1))) & mask;
      uint8_t *px = row_out + 3 * (x0 + dx * xp);
      if (ct == 3) {
        const uint32_t e = cv.pal[v];
        put_bgr(px, e & 0xFFu, (e >> 8) & 0xFFu, (e >> 16) & 0xFFu);
      } else {
        const uint32_t g = (cv.has_key && v == cv.key[0]) ? 0u : v * (255u / mask);
        put_bgr(px, g, g, g);
      }
    }
    return;
  }
  uint8_t *px = row_out + 3 * (x0 + dx * x);
  auto byte = [&](int i) { return (uint32_t)((u >> (8 * i)) & 0xFFu); };
  if (d == 16) {  // OpenCV: the high byte of each sample, alpha dropped
    if (ct == 0 || ct == 4) put_bgr(px, byte(0), byte(0), byte(0));
    else put_bgr(px, byte(4), byte(2), byte(0));
    return;
  }
  switch (ct) {
    case 0: {
      const uint32_t g = (cv.has_key && byte(0) == cv.key[0]) ? 0u : byte(0);
      put_bgr(px, g, g, g);
      break;
    }
    case 2: {
      const bool k = cv.has_key && byte(0) == cv.key[0] && byte(1) == cv.key[1] &&
                     byte(2) == cv.key[2];
      if (k) put_bgr(px, 0, 0, 0);
      else put_bgr(px, byte(2), byte(1), byte(0));
      break;
    }
    case 3: {
      const uint32_t e = cv.pal[byte(0)];
      put_bgr(px, e & 0xFFu, (e >> 8) & 0xFFu, (e >> 16) & 0xFFu);
      break;
    }
    case 4: {
      const uint32_t g = premul(byte(0), byte(1));
      put_bgr(px, g, g, g);
      break;
    }
    default: {  // 6
      const uint32_t a = byte(3);
      put_bgr(px, premul(byte(2), a), premul(byte(1), a), premul(byte(0), a));
      break;
    }
  }
}

// One pass (or the whole non-interlaced image). Returns kBadFilter on a
// filter type above 4. Rows go in groups of 32, lane k on row r0 + k, one
// unit behind lane k - 1; lane 31 writes its reconstructed row back over the
// scanline buffer so that the next group's lane 0 can read it as "above".
template <int BPP>
__device__ int unfilter_pass(uint8_t *raw, int64_t pw, int64_t ph, int64_t rowbytes,
                             const Conv &cv, uint8_t *dst, uint64_t pitch, int x0, int y0, int dx,
                             int dy, int lane) {
  const int64_t units = rowbytes / BPP;  // exact: rowbytes is a multiple of BPP
  const int64_t stride = rowbytes + 1;
  int bad = 0;
  for (int64_t r0 = 0; r0 < ph; r0 += 32) {
    const int64_t r = r0 + lane;
    const bool active = r < ph;
    uint8_t *row = raw + r * stride;
    const uint32_t ft = active ? row[0] : 0u;
    if (active && ft > 4) bad = 1;
    const uint8_t *above0 = r0 > 0 ? raw + (r0 - 1) * stride + 1 : nullptr;  // lane 0's row above
    uint8_t *row_out = dst + (uint64_t)(y0 + dy * r) * pitch;
    uint64_t cur = 0, prev_b = 0;
    const int64_t steps = units + 31;
    for (int64_t t = 0; t < steps; ++t) {
      const uint64_t from_above = __shfl_up_sync(kFull, cur, 1);
      const int64_t j = t - lane;
      if (active && j >= 0 && j < units) {
        uint64_t b = from_above;
        if (lane == 0) {
          b = 0;
          if (above0)
#pragma unroll
            for (int i = 0; i < BPP; ++i) b |= uint64_t(above0[j * BPP + i]) << (8 * i);
        }
        const uint64_t a = j > 0 ? cur : 0, c = j > 0 ? prev_b : 0;
        const uint8_t *fp = row + 1 + j * BPP;
        uint64_t nu = 0;
#pragma unroll
        for (int i = 0; i < BPP; ++i) {
          const uint32_t ai = (a >> (8 * i)) & 0xFFu, bi = (b >> (8 * i)) & 0xFFu,
                         ci = (c >> (8 * i)) & 0xFFu;
          uint32_t pred = 0;
          if (ft == 1) pred = ai;
          else if (ft == 2) pred = bi;
          else if (ft == 3) pred = (ai + bi) >> 1;
          else if (ft == 4) pred = paeth(ai, bi, ci);
          nu |= uint64_t((fp[i] + pred) & 0xFFu) << (8 * i);
        }
        cur = nu;
        prev_b = b;
        if (lane == 31)
#pragma unroll
          for (int i = 0; i < BPP; ++i) row[1 + j * BPP + i] = (uint8_t)(nu >> (8 * i));
        emit_unit<BPP>(cv, nu, j, pw, row_out, x0, dx);
      }
    }
    __syncwarp();
  }
  return __any_sync(kFull, bad) ? kBadFilter : kOk;
}

template <int BPP>
__device__ int unfilter_image(uint8_t *raw, const Meta &m, const Conv &cv, int64_t W, int64_t H,
                              uint8_t *dst, uint64_t pitch, int lane) {
  const int ch = channels_of(m.ctype);
  uint64_t off = 0;
  int st = kOk;
  for (int p = 0; p < (m.interlace ? 7 : 1) && st == kOk; ++p) {
    int x0, y0, dx, dy;
    pass_geom(m.interlace, p, x0, y0, dx, dy);
    const int64_t pw = W > x0 ? (W - x0 + dx - 1) / dx : 0;
    const int64_t ph = H > y0 ? (H - y0 + dy - 1) / dy : 0;
    if (!pw || !ph) continue;
    const int64_t rb = (int64_t)row_bytes(pw, ch, m.depth);
    st = unfilter_pass<BPP>(raw + off, pw, ph, rb, cv, dst, pitch, x0, y0, dx, dy, lane);
    off += (uint64_t)ph * (rb + 1);
  }
  return st;
}

// ---- tiled unfilter: one CTA per image, kTW warps on consecutive row groups ----
// Non-interlaced files of 8 / 16 bit samples and at most 4 bytes per pixel
// (every colour type at depth 8, grey and grey+alpha at 16). Each warp runs
// the same wavefront as unfilter_pass over its group of 32 rows, but reads
// the filtered bytes from shared memory: tiles of 32 units x 33 rows (the
// group's rows and the reconstructed row above it) are fetched with
// cp.async one window ahead, and the BGR pixels go through a shared tile so
// that they leave in coalesced 4-byte stores. Group g + 1 reads group g's
// last row once the warp of group g has published, in shared memory, how
// many of its units are written back (bounded wait).
constexpr int kTW = 8;
constexpr int kTU = 32;
constexpr int kTileRow = 32 * 4 + 16;  // bytes of one tile row in shared memory (BPP <= 4)
constexpr long long kSpinLimit = 1ll << 24;

struct alignas(16) TileWarp {
  uint8_t in[3][33][kTileRow];
  uint8_t out[2][32][96];
  uint8_t mis[3][33];  // byte offset of the tile's first byte inside its row buffer
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Pixel of one 8/16-bit unit into the shared output tile (3 bytes).
template <int BPP>
__device__ __forceinline__ void emit_px(const Conv &cv, uint64_t u, uint8_t *o) {
  auto byte = [&](int i) { return (uint32_t)((u >> (8 * i)) & 0xFFu); };
  uint32_t b, g, r;
  if (cv.depth == 16) {
    if (BPP == 6 || BPP == 8) { b = byte(4); g = byte(2); r = byte(0); }
    else { b = g = r = byte(0); }
  } else if (cv.ctype == 0) {
    b = g = r = (cv.has_key && byte(0) == cv.key[0]) ? 0u : byte(0);
  } else if (cv.ctype == 2) {
    const bool k = cv.has_key && byte(0) == cv.key[0] && byte(1) == cv.key[1] && byte(2) == cv.key[2];
    b = k ? 0u : byte(2); g = k ? 0u : byte(1); r = k ? 0u : byte(0);
  } else if (cv.ctype == 3) {
    const uint32_t e = cv.pal[byte(0)];
    b = e & 0xFFu; g = (e >> 8) & 0xFFu; r = (e >> 16) & 0xFFu;
  } else if (cv.ctype == 4) {
    b = g = r = premul(byte(0), byte(1));
  } else {
    const uint32_t a = byte(3);
    b = premul(byte(2), a); g = premul(byte(1), a); r = premul(byte(0), a);
  }
  o[0] = (uint8_t)b; o[1] = (uint8_t)g; o[2] = (uint8_t)r;
}

template <int BPP>
__device__ int unfilter_tiled(uint8_t *raw, int64_t W, int64_t H, const Conv &cv, uint8_t *dst,
                              uint64_t pitch, TileWarp &T, volatile unsigned long long *prog,
                              int warp, int lane) {
  const int64_t units = W, stride = W * BPP + 1;
  const int64_t ngroups = (H + 31) / 32, ntiles = (units + kTU - 1) / kTU;
  const unsigned long long gspan = (unsigned long long)units + 1;  // progress per group
  constexpr int TB = kTU * BPP, NV = (TB + 16) / 16;
  const bool out4 = ((reinterpret_cast<uintptr_t>(dst) | pitch) & 3u) == 0;
  int bad = 0;
  for (int64_t g = warp; g < ngroups; g += kTW) {
    const int64_t r0 = g * 32;
    const bool active = r0 + lane < H, has_next = g + 1 < ngroups;
    const uint32_t ft = active ? raw[(r0 + lane) * stride] : 0u;
    if (active && ft > 4) bad = 1;
    // Tile m of the group's rows (and of the row above) into slot m % 3.
    auto load_tile = [&](int64_t m) {
      if (m >= ntiles) return;
      const int slot = (int)(m % 3);
      if (g > 0) {  // the row above must be written back up to this tile's end
        const unsigned long long need =
            (unsigned long long)(g - 1) * gspan +
            (unsigned long long)(units < (m + 1) * kTU ? units : (m + 1) * kTU);
        if (lane == 0) {
          long long spins = 0;
          while (prog[(g - 1) % kTW] < need && ++spins < kSpinLimit) __nanosleep(64);
          if (spins >= kSpinLimit) bad = 2;
        }
        __syncwarp();
        __threadfence();
      }
      for (int idx = lane; idx < 33 * NV; idx += 32) {
        const int i = idx / NV, v = idx % NV;
        const int64_t row = i < 32 ? r0 + i : r0 - 1;
        if ((i < 32 && row >= H) || (i == 32 && g == 0)) continue;
        const int64_t sb = row * stride + 1 + m * TB, a = sb & ~15ll;
        if (v == 0) T.mis[slot][i] = (uint8_t)(sb - a);
        cp_async16(&T.in[slot][i][16 * v], raw + a + 16 * v);
      }
      cp_async_commit();
    };
    auto flush = [&](int64_t m) {
      const int slot = (int)(m & 1);
      const int64_t x0 = m * kTU;
      const int64_t rem = units - x0;
      const int nb = 3 * (int)(rem < kTU ? rem : kTU);
      __syncwarp();
      if (out4) {
        const int nw = (nb + 3) / 4;
        for (int idx = lane; idx < 32 * 24; idx += 32) {
          const int i = idx / 24, k = idx % 24;
          if (k >= nw || r0 + i >= H) continue;
          uint8_t *o = dst + (uint64_t)(r0 + i) * pitch + 3 * x0 + 4 * k;
          const uint8_t *sp = &T.out[slot][i][4 * k];
          if (4 * k + 4 <= nb) *reinterpret_cast<uint32_t *>(o) = *reinterpret_cast<const uint32_t *>(sp);
          else for (int q = 0; 4 * k + q < nb; ++q) o[q] = sp[q];
        }
      } else {
        for (int idx = lane; idx < 32 * 96; idx += 32) {
          const int i = idx / 96, k = idx % 96;
          if (k < nb && r0 + i < H) dst[(uint64_t)(r0 + i) * pitch + 3 * x0 + k] = T.out[slot][i][k];
        }
      }
      __syncwarp();
    };
    load_tile(0);
    uint64_t cur = 0, prev_b = 0;
    int64_t flushed = 0;  // output tiles already stored
    const int64_t steps = units + 31;
    for (int64_t t = 0; t < steps; ++t) {
      if ((t & 31) == 0) {
        const int64_t w = t >> 5;
        cp_async_wait_all();
        __syncwarp();
        if (has_next) {  // lane 31's row: units < 32w - 31 are written back
          int64_t done = 32 * w - 31;
          done = done < 0 ? 0 : done > units ? units : done;
          if (lane == 31) {
            __threadfence();
            prog[g % kTW] = (unsigned long long)g * gspan + (unsigned long long)done;
          }
        }
        while (flushed < w - 1) flush(flushed++);
        load_tile(w + 1);
      }
      const uint64_t from_above = __shfl_up_sync(kFull, cur, 1);
      const int64_t j = t - lane;
      if (active && j >= 0 && j < units) {
        const int64_t m = j / kTU;
        const int slot = (int)(m % 3), col = (int)(j - m * kTU);
        const uint8_t *fp = &T.in[slot][lane][T.mis[slot][lane] + col * BPP];
        uint64_t b = from_above;
        if (lane == 0) {
          b = 0;
          if (g > 0) {
            const uint8_t *ap = &T.in[slot][32][T.mis[slot][32] + col * BPP];
#pragma unroll
            for (int i = 0; i < BPP; ++i) b |= uint64_t(ap[i]) << (8 * i);
          }
        }
        const uint64_t a = j > 0 ? cur : 0, c = j > 0 ? prev_b : 0;
        uint64_t nu = 0;
#pragma unroll
        for (int i = 0; i < BPP; ++i) {
          const uint32_t ai = (a >> (8 * i)) & 0xFFu, bi = (b >> (8 * i)) & 0xFFu,
                         ci = (c >> (8 * i)) & 0xFFu;
          uint32_t pred = 0;
          if (ft == 1) pred = ai;
          else if (ft == 2) pred = bi;
          else if (ft == 3) pred = (ai + bi) >> 1;
          else if (ft == 4) pred = paeth(ai, bi, ci);
          nu |= uint64_t((fp[i] + pred) & 0xFFu) << (8 * i);
        }
        cur = nu;
        prev_b = b;
        if (lane == 31 && has_next) {
          uint8_t *wb = raw + (r0 + 31) * stride + 1 + j * BPP;
#pragma unroll
          for (int i = 0; i < BPP; ++i) wb[i] = (uint8_t)(nu >> (8 * i));
        }
        emit_px<BPP>(cv, nu, &T.out[m & 1][lane][3 * col]);
      }
    }
    while (flushed < ntiles) flush(flushed++);
    cp_async_wait_all();
    if (has_next && lane == 31) {
      __threadfence();
      prog[g % kTW] = (unsigned long long)g * gspan + (unsigned long long)units;
    }
    __syncwarp();
  }
  return bad;  // per lane; the caller reduces
}

__global__ void __launch_bounds__(kTW * 32)
png_unfilter_kernel(const uint8_t *__restrict__ src, const tocr_png_job *__restrict__ jobs, int n,
                    uint8_t *__restrict__ dst, uint8_t *__restrict__ scratch,
                    int32_t *__restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem_unf[];
  __shared__ uint32_t s_pal[256];
  __shared__ volatile unsigned long long s_prog[kTW];
  __shared__ int s_bad;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int img = blockIdx.x;
  const tocr_png_job job = jobs[img];
  uint8_t *base = scratch + job.scratch_off;
  const Meta m = *reinterpret_cast<const Meta *>(base);
  if (m.status != kOk) {
    if (threadIdx.x == 0) status[img] = m.status;
    return;
  }
  const uint8_t *f = src + job.src_off;
  Conv cv;
  cv.ctype = m.ctype;
  cv.depth = m.depth;
  cv.pal = s_pal;
  cv.has_key = false;
  cv.key[0] = cv.key[1] = cv.key[2] = 0;
  if (m.ctype == 3) {
    // PLTE (+ tRNS alphas) premultiplied as Wuffs does; entries past the
    // PLTE are opaque black.
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      uint32_t e = 0;
      if ((uint32_t)i * 3 < m.plte_len) {
        const uint8_t *pe = f + m.plte_pos + 3 * i;
        const uint32_t a = (uint32_t)i < m.trns_len ? f[m.trns_pos + i] : 255u;
        e = premul(pe[2], a) | (premul(pe[1], a) << 8) | (premul(pe[0], a) << 16);
      }
      s_pal[i] = e;
    }
  } else if (m.trns_len && m.depth <= 8) {
    // Colour types 0 and 2: the key's samples, low `depth` bits compared.
    const uint32_t mask = (1u << m.depth) - 1u;
    cv.has_key = true;
    for (int c = 0; c < (m.ctype == 2 ? 3 : 1); ++c)
      cv.key[c] = (uint32_t)(f[m.trns_pos + 2 * c + 1]) & mask;
  }
  if (threadIdx.x < kTW) s_prog[threadIdx.x] = 0;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const int bpp = max(1, channels_of(m.ctype) * m.depth / 8);
  uint8_t *raw = base + kMetaBytes;
  uint8_t *out = dst + job.dst_off;
  int st = kOk;
  if (!m.interlace && m.depth >= 8 && bpp <= 4) {
    TileWarp &T = reinterpret_cast<TileWarp *>(smem_unf)[warp];
    int bad = 0;
    switch (bpp) {
      case 1: bad = unfilter_tiled<1>(raw, job.width, job.height, cv, out, job.dst_pitch, T, s_prog, warp, lane); break;
      case 2: bad = unfilter_tiled<2>(raw, job.width, job.height, cv, out, job.dst_pitch, T, s_prog, warp, lane); break;
      case 3: bad = unfilter_tiled<3>(raw, job.width, job.height, cv, out, job.dst_pitch, T, s_prog, warp, lane); break;
      default: bad = unfilter_tiled<4>(raw, job.width, job.height, cv, out, job.dst_pitch, T, s_prog, warp, lane); break;
    }
    if (bad) atomicMax(&s_bad, bad);
    __syncthreads();
    st = s_bad == 2 ? kTimeout : s_bad ? kBadFilter : kOk;
  } else if (warp == 0) {
    switch (bpp) {
      case 1: st = unfilter_image<1>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
      case 2: st = unfilter_image<2>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
      case 3: st = unfilter_image<3>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
      case 4: st = unfilter_image<4>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
      case 6: st = unfilter_image<6>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
      default: st = unfilter_image<8>(raw, m, cv, job.width, job.height, out, job.dst_pitch, lane); break;
    }
  }
  if (threadIdx.x == 0) status[img] = st;
}

}  // namespace png
}  // namespace tocr

// ---- C-ABI ----
extern "C" {

TOCR_API int tocr_png_peek(const uint8_t *data, size_t len, int max_dim, long long max_pixels,
                           tocr_png_info *info) {
  using namespace tocr::png;
  TOCR_REQUIRE(info != nullptr, "tocr_png_peek: null info");
  std::memset(info, 0, sizeof *info);
  TOCR_REQUIRE(data != nullptr || len == 0, "tocr_png_peek: null data");
  static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
  TOCR_REQUIRE(len >= 33 && std::memcmp(data, sig, 8) == 0 && be32(data + 8) == 13 &&
                   be32(data + 12) == kIHDR,
               "tocr_png_peek: not a PNG (signature / IHDR)");
  const uint32_t w = be32(data + 16), h = be32(data + 20);
  const int depth = data[24], ct = data[25], il = data[28];
  info->width = (int32_t)(w > 0x7FFFFFFFu ? 0x7FFFFFFF : w);
  info->height = (int32_t)(h > 0x7FFFFFFFu ? 0x7FFFFFFF : h);
  info->bit_depth = depth;
  info->color_type = ct;
  info->interlace = il;
  TOCR_REQUIRE(w > 0 && h > 0 && w <= 16777215u && h <= 16777215u,
               "tocr_png_peek: dimensions %ux%u out of range", w, h);
  TOCR_REQUIRE(depth_ok(ct, depth) && data[26] == 0 && data[27] == 0 && il <= 1,
               "tocr_png_peek: unsupported IHDR (depth %d, colour type %d)", depth, ct);
  TOCR_REQUIRE(max_dim > 0 && w <= (uint32_t)max_dim && h <= (uint32_t)max_dim,
               "tocr_png_peek: dimensions %ux%u exceed the %d cap", w, h, max_dim);
  TOCR_REQUIRE((long long)w * (long long)h <= max_pixels,
               "tocr_png_peek: %ux%u exceeds the %lld pixel cap", w, h, max_pixels);
  info->raw_bytes = raw_size(w, h, ct, depth, il);
  info->scratch_bytes = scratch_size(info->raw_bytes, len);
  return TOCR_OK;
}

TOCR_API int tocr_png_decode_batch(const uint8_t *d_src, const tocr_png_job *d_jobs, int n,
                                   uint8_t *d_dst, uint8_t *d_scratch, int32_t *d_status,
                                   void *stream) {
  using namespace tocr;
  using namespace tocr::png;
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && n <= (1 << 24), "tocr_png_decode_batch: bad n=%d", n);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_src && d_jobs && d_dst && d_scratch && d_status,
               "tocr_png_decode_batch: null pointer");
  TOCR_REQUIRE(aligned(d_scratch, 16), "tocr_png_decode_batch: scratch not 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  png_parse_kernel<<<(n + kParseWarps - 1) / kParseWarps, kParseWarps * 32, 0, s>>>(d_src, d_jobs,
                                                                                  n, d_scratch);
  int st = check_launch("png_parse_kernel");
  if (st) return st;
  const size_t smem = sizeof(InflateImg) * kInfImgs;
  if (cudaFuncSetAttribute(png_inflate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return check_launch("png_inflate_kernel (shared memory attribute)");
  png_inflate_kernel<<<(n + kInfImgs - 1) / kInfImgs, kInfImgs * 64, smem, s>>>(d_src, d_jobs, n,
                                                                               d_scratch);
  st = check_launch("png_inflate_kernel");
  if (st) return st;
  const size_t smem_u = sizeof(TileWarp) * kTW;
  if (cudaFuncSetAttribute(png_unfilter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem_u) != cudaSuccess)
    return check_launch("png_unfilter_kernel (shared memory attribute)");
  png_unfilter_kernel<<<n, kTW * 32, smem_u, s>>>(d_src, d_jobs, n, d_dst, d_scratch, d_status);
  return check_launch("png_unfilter_kernel");
}

}  // extern "C"
