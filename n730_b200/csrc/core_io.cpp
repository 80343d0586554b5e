// .n730 file reader and host dequant: the reference's n730core C ABI
// (src-code/cpp/n730core.cpp, bound by src-code/scheduler.py:56-84), rebuilt.
//
// Same symbols, arguments, and error codes (-1 BAD_MAGIC, -2 FILE, -3 ALLOC,
// -4 BAD_LAYER, -5 BAD_PREC, -6 NULL; n730core.cpp:22-28).  Differences:
//  * pread() on a file descriptor instead of a shared FILE* position, so
//    concurrent readers of one handle are safe (the reference handle is not,
//    scheduler.py:242-244);
//  * per-tensor dequant goes through a 2^bits-entry lookup table whose entries
//    are computed with the reference formula ((float)q - zp) * scale, so the
//    output is bit-identical while the loop is a gather;
//  * the group-wise precision ids (0x42/0x44/0x48) are decoded as well;
//  * n730_read_block returns a block's header fields and raw payload without
//    dequantising (used to upload packed codes to the GPU).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#define N730_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int OK = 0, ERR_BAD_MAGIC = -1, ERR_FILE = -2, ERR_ALLOC = -3, ERR_BAD_LAYER = -4,
              ERR_BAD_PREC = -5, ERR_NULL = -6;
constexpr uint8_t FILE_MAGIC[8] = {'N', '7', '3', '0', 0, 1, 0, 0};
constexpr uint8_t LAYER_MAGIC[4] = {'L', 'Y', 'R', 0};
constexpr int HDR = 29;

struct Handle {
  int fd;
  int64_t size;
};

inline uint32_t be32(const uint8_t* p) {
  return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3];
}
inline float befloat(const uint8_t* p) {
  uint32_t u = be32(p);
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// IEEE binary16 -> binary32, exact.
inline float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FFu, bits;
  if (e == 0) {
    if (m == 0) bits = sign;
    else {
      int s = 0;
      while (!(m & 0x400u)) { m <<= 1; ++s; }
      bits = sign | ((uint32_t)(113 - s) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (m << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

inline int bits_of(int prec) {
  switch (prec) {
    case 2: case 0x42: return 2;
    case 4: case 0x44: return 4;
    case 8: case 0x48: return 8;
    case 16: return 16;
  }
  return 0;
}

struct BlockHdr {
  uint32_t idx, rows, cols, data_size;
  int prec;
  float scale, zp;
};

int read_hdr(const Handle* h, int64_t off, BlockHdr* b) {
  uint8_t buf[HDR];
  if (off < 0 || pread(h->fd, buf, HDR, off) != HDR) return ERR_FILE;
  if (memcmp(buf, LAYER_MAGIC, 4) != 0) return ERR_BAD_LAYER;
  b->idx = be32(buf + 4);
  b->prec = buf[8];
  b->rows = be32(buf + 9);
  b->cols = be32(buf + 13);
  b->scale = befloat(buf + 17);
  b->zp = befloat(buf + 21);
  b->data_size = be32(buf + 25);
  return OK;
}

// Per-tensor dequant with the reference formula, through a lookup table.
void dequant_tensor(const uint8_t* src, float* dst, int64_t n, int bits, float scale, float zp) {
  const int nv = 1 << bits;
  float lut[256];
  for (int q = 0; q < nv; ++q) {
    volatile float d = (float)q - zp;  // keep the subtraction rounded on its own
    lut[q] = d * scale;
  }
  if (bits == 8) {
    for (int64_t i = 0; i < n; ++i) dst[i] = lut[src[i]];
  } else if (bits == 4) {
    int64_t i = 0;
    for (; i + 1 < n; i += 2) {
      const uint8_t b = src[i >> 1];
      dst[i] = lut[b & 15];
      dst[i + 1] = lut[b >> 4];
    }
    if (i < n) dst[i] = lut[src[i >> 1] & 15];
  } else {
    for (int64_t i = 0; i < n; ++i) dst[i] = lut[(src[i >> 2] >> (2 * (i & 3))) & 3];
  }
}

int dequant_grouped(const uint8_t* payload, int64_t data_size, int bits, int64_t rows, int64_t cols,
                    float* dst) {
  const int64_t code_bytes = (rows * cols * bits + 7) / 8;
  const int64_t extra = data_size - code_bytes;
  if (extra <= 0 || extra % (4 * rows)) return ERR_BAD_LAYER;
  const int64_t G = extra / (4 * rows);
  if (G <= 0 || cols % G) return ERR_BAD_LAYER;
  const int64_t g = cols / G;
  const uint16_t* s16 = (const uint16_t*)(payload + code_bytes);
  const uint16_t* z16 = s16 + rows * G;
  const int nv = 1 << bits;
  float lut[256];
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t gi = 0; gi < G; ++gi) {
      uint16_t sh, zh;
      memcpy(&sh, s16 + r * G + gi, 2);
      memcpy(&zh, z16 + r * G + gi, 2);
      const float s = half_to_float(sh), z = half_to_float(zh);
      for (int q = 0; q < nv; ++q) {
        volatile float d = (float)q - z;
        lut[q] = d * s;
      }
      const int64_t e0 = r * cols + gi * g;
      for (int64_t c = 0; c < g; ++c) {
        const int64_t e = e0 + c;
        uint32_t q;
        if (bits == 8) q = payload[e];
        else if (bits == 4) q = (payload[e >> 1] >> (4 * (e & 1))) & 15;
        else q = (payload[e >> 2] >> (2 * (e & 3))) & 3;
        dst[e] = lut[q];
      }
    }
  return OK;
}

}  // namespace

N730_API int64_t n730_open(const char* path) {
  if (!path) return ERR_NULL;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return ERR_FILE;
  uint8_t magic[8];
  if (pread(fd, magic, 8, 0) != 8 || memcmp(magic, FILE_MAGIC, 8) != 0) {
    close(fd);
    return ERR_BAD_MAGIC;
  }
  struct stat st;
  fstat(fd, &st);
  Handle* h = new (std::nothrow) Handle{fd, (int64_t)st.st_size};
  if (!h) { close(fd); return ERR_ALLOC; }
  return (int64_t)(uintptr_t)h;
}

N730_API void n730_close(int64_t handle) {
  Handle* h = (Handle*)(uintptr_t)handle;
  if (handle > 0 && h) {
    close(h->fd);
    delete h;
  }
}

N730_API int32_t n730_read_layer(int64_t handle, int64_t file_offset, float* out, int32_t* out_rows,
                                 int32_t* out_cols, int32_t* out_prec) {
  if (handle <= 0 || !out) return ERR_NULL;
  const Handle* h = (const Handle*)(uintptr_t)handle;
  BlockHdr b;
  if (int rc = read_hdr(h, file_offset, &b)) return rc;
  if (out_rows) *out_rows = (int32_t)b.rows;
  if (out_cols) *out_cols = (int32_t)b.cols;
  if (out_prec) *out_prec = b.prec;
  const int bits = bits_of(b.prec);
  if (!bits) return ERR_BAD_PREC;
  std::vector<uint8_t> raw;
  try { raw.resize(b.data_size); } catch (...) { return ERR_ALLOC; }
  if (b.data_size && pread(h->fd, raw.data(), b.data_size, file_offset + HDR) != (ssize_t)b.data_size)
    return ERR_FILE;
  const int64_t n = (int64_t)b.rows * b.cols;
  if (b.prec == 16) {
    if ((int64_t)b.data_size < 2 * n) return ERR_BAD_LAYER;
    for (int64_t i = 0; i < n; ++i) {
      uint16_t v;
      memcpy(&v, raw.data() + 2 * i, 2);
      out[i] = half_to_float(v);
    }
    return OK;
  }
  if (b.prec & 0x40) return dequant_grouped(raw.data(), b.data_size, bits, b.rows, b.cols, out);
  // per-tensor: decode what the block holds, as the reference does (it reads
  // data_size bytes and unpacks the first rows*cols codes)
  const int64_t have = (int64_t)b.data_size * 8 / bits;
  dequant_tensor(raw.data(), out, n < have ? n : have, bits, b.scale, b.zp);
  for (int64_t i = have; i < n; ++i) out[i] = ((float)0 - b.zp) * b.scale;
  return OK;
}

// Header fields and raw payload of one block, no dequant.
// hdr[0..7] = layer_idx, prec_id, rows, cols, data_size, group_size (0 if per-tensor),
//             scale bits, zero-point bits (float32 bit patterns).
N730_API int32_t n730_read_block(int64_t handle, int64_t file_offset, int64_t* hdr, uint8_t* payload,
                                 int64_t capacity) {
  if (handle <= 0 || !hdr) return ERR_NULL;
  const Handle* h = (const Handle*)(uintptr_t)handle;
  BlockHdr b;
  if (int rc = read_hdr(h, file_offset, &b)) return rc;
  const int bits = bits_of(b.prec);
  if (!bits) return ERR_BAD_PREC;
  int64_t group = 0;
  if (b.prec & 0x40) {
    const int64_t code_bytes = ((int64_t)b.rows * b.cols * bits + 7) / 8;
    const int64_t extra = (int64_t)b.data_size - code_bytes;
    if (extra <= 0 || extra % (4 * (int64_t)b.rows)) return ERR_BAD_LAYER;
    const int64_t G = extra / (4 * (int64_t)b.rows);
    if (b.cols % G) return ERR_BAD_LAYER;
    group = b.cols / G;
  }
  uint32_t sb, zb;
  memcpy(&sb, &b.scale, 4);
  memcpy(&zb, &b.zp, 4);
  hdr[0] = b.idx; hdr[1] = b.prec; hdr[2] = b.rows; hdr[3] = b.cols; hdr[4] = b.data_size;
  hdr[5] = group; hdr[6] = sb; hdr[7] = zb;
  if (!payload) return OK;  // header probe only
  if (capacity < (int64_t)b.data_size) return ERR_ALLOC;
  if (b.data_size && pread(h->fd, payload, b.data_size, file_offset + HDR) != (ssize_t)b.data_size)
    return ERR_FILE;
  return OK;
}

N730_API int32_t n730_layer_elements(int64_t handle, int64_t file_offset) {
  if (handle <= 0) return ERR_NULL;
  BlockHdr b;
  if (int rc = read_hdr((const Handle*)(uintptr_t)handle, file_offset, &b)) return rc;
  return (int32_t)((int64_t)b.rows * b.cols);
}

N730_API int32_t n730_probe_layer_size(int64_t handle, int64_t file_offset) {
  return n730_layer_elements(handle, file_offset);
}

N730_API const char* n730_version() { return "N730 core (B200 build) 0.1"; }
