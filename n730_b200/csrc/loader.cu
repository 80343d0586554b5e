// Native .n730 block loader: packed weights from the file to HBM without a
// Python read per tensor.
//
// The reference reads each weight's raw bytes in Python for every use
// (src-code/inference.py:355-366) or reads and dequantises a block in its C core
// (src-code/cpp/n730core.cpp:192-248).  Here a block goes once from the file
// into HBM, still packed:
//  * a pre-pass reads every requested block header (29 bytes, big-endian
//    ">4sIBIIffi", n730core.cpp:144-155), validates magic, precision id and
//    payload size, and sizes the staging buffers to the largest payload;
//  * two page-aligned pinned host buffers and two device staging buffers
//    alternate: block i is read with pread straight into pinned memory (no
//    intermediate copy) while block i-1's asynchronous host->device copy and
//    its conversion into the weight's own layout (qweight_create from device
//    memory) run on the stream; an event per buffer guards its reuse.
// Per-tensor ids 2/4/8/16 and the group-wise ids 0x42/0x44/0x48 are accepted.
// (An odd-length per-tensor INT4/INT2 block written through the reference's
// int64 packing quirk has a larger payload than its codes; such blocks are
// rejected here and left to the Python reader, which decodes them.)
#include <fcntl.h>
#include <unistd.h>

#include <cstring>
#include <vector>

#include "qweight.h"

namespace n730 {

int qweight_create(int prec, int rows, int cols, int group, float scale, float zp, const void* codes,
                   const void* s16, const void* z16, bool src_device, cudaStream_t st, QWeight** out);
void qweight_destroy(QWeight* w);

struct BlockHdr {
  int prec = 0, rows = 0, cols = 0, group = 0;
  float scale = 1.f, zp = 0.f;
  int64_t payload = 0, codes = 0;
};

static uint32_t be32(const uint8_t* p) { return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]; }
static float bef(const uint8_t* p) {
  const uint32_t u = be32(p);
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static bool read_full(int fd, void* buf, size_t n, int64_t off) {
  uint8_t* b = static_cast<uint8_t*>(buf);
  while (n) {
    const ssize_t r = pread(fd, b, n, (off_t)off);
    if (r <= 0) return false;
    b += r;
    n -= (size_t)r;
    off += r;
  }
  return true;
}

static int parse_block(int fd, int64_t off, BlockHdr* h) {
  uint8_t raw[29];
  N730_REQUIRE(off >= 0 && read_full(fd, raw, sizeof raw, off), N730_BAD_ARG,
               "load_blocks: cannot read a block header at offset %lld", (long long)off);
  N730_REQUIRE(memcmp(raw, "LYR\0", 4) == 0, N730_BAD_ARG, "load_blocks: bad layer magic at offset %lld",
               (long long)off);
  h->prec = raw[8];
  h->rows = (int)be32(raw + 9);
  h->cols = (int)be32(raw + 13);
  h->scale = bef(raw + 17);
  h->zp = bef(raw + 21);
  h->payload = (int32_t)be32(raw + 25);
  const int bits = prec_bits(h->prec);
  N730_REQUIRE(bits, N730_BAD_ARG, "load_blocks: unknown precision id %d at offset %lld", h->prec, (long long)off);
  N730_REQUIRE(h->rows > 0 && h->cols > 0 && h->payload > 0, N730_BAD_ARG, "load_blocks: bad block sizes at %lld",
               (long long)off);
  h->codes = ((int64_t)h->rows * h->cols * bits + 7) / 8;
  if (prec_grouped(h->prec)) {
    const int64_t extra = h->payload - h->codes;
    N730_REQUIRE(extra > 0 && extra % (4ll * h->rows) == 0, N730_BAD_ARG,
                 "load_blocks: grouped block sizes inconsistent at %lld", (long long)off);
    const int64_t G = extra / (4ll * h->rows);
    N730_REQUIRE(G > 0 && h->cols % G == 0, N730_BAD_ARG, "load_blocks: %lld groups do not divide %d columns",
                 (long long)G, h->cols);
    h->group = (int)(h->cols / G);
  } else {
    N730_REQUIRE(h->payload == h->codes, N730_UNSUPPORTED,
                 "load_blocks: per-tensor block at %lld holds %lld bytes for %lld code bytes (left to the Python reader)",
                 (long long)off, (long long)h->payload, (long long)h->codes);
  }
  return N730_OK;
}

int load_blocks(const char* path, int n, const int64_t* offsets, cudaStream_t st, QWeight** out, int64_t* bytes) {
  N730_REQUIRE(path && offsets && out && n >= 0, N730_NULL, "load_blocks: null argument");
  for (int i = 0; i < n; ++i) out[i] = nullptr;
  if (bytes) *bytes = 0;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  N730_REQUIRE(fd >= 0, N730_BAD_ARG, "load_blocks: cannot open %s", path);
  std::vector<BlockHdr> hdr((size_t)n);
  int64_t max_payload = 16;
  for (int i = 0; i < n; ++i) {
    if (int rc = parse_block(fd, offsets[i], &hdr[i])) { close(fd); return rc; }
    max_payload = std::max(max_payload, hdr[i].payload);
  }
  uint8_t* pin[2] = {nullptr, nullptr};
  uint8_t* dev[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  int rc = N730_OK;
  int64_t total = 0;
  auto cleanup = [&]() {
    cudaStreamSynchronize(st);
    for (int b = 0; b < 2; ++b) {
      if (pin[b]) cudaFreeHost(pin[b]);
      if (dev[b]) cudaFree(dev[b]);
      if (ev[b]) cudaEventDestroy(ev[b]);
    }
    close(fd);
  };
  for (int b = 0; b < 2 && !rc; ++b) {
    if (cudaHostAlloc((void**)&pin[b], (size_t)max_payload, cudaHostAllocDefault) != cudaSuccess ||
        cudaMalloc((void**)&dev[b], (size_t)max_payload) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      set_error("load_blocks: staging allocation of 2 x %lld bytes failed", (long long)max_payload);
      rc = N730_OOM;
    }
  }
  for (int i = 0; i < n && !rc; ++i) {
    const int b = i & 1;
    const BlockHdr& h = hdr[i];
    if ((rc = cuda_rc(cudaEventSynchronize(ev[b]), __FILE__, __LINE__))) break;  // buffer b's last copy is done
    if (!read_full(fd, pin[b], (size_t)h.payload, offsets[i] + 29)) {
      set_error("load_blocks: short read of block at offset %lld", (long long)offsets[i]);
      rc = N730_BAD_ARG;
      break;
    }
    total += 29 + h.payload;
    if ((rc = cuda_rc(cudaMemcpyAsync(dev[b], pin[b], (size_t)h.payload, cudaMemcpyHostToDevice, st), __FILE__,
                      __LINE__)))
      break;
    const uint8_t* s16 = nullptr;
    const uint8_t* z16 = nullptr;
    if (h.group) {
      const int64_t ng = (int64_t)h.rows * (h.cols / h.group);
      s16 = dev[b] + h.codes;
      z16 = s16 + 2 * ng;
    }
    if ((rc = qweight_create(h.prec, h.rows, h.cols, h.group, h.scale, h.zp, dev[b], s16, z16, true, st, &out[i])))
      break;
    if ((rc = cuda_rc(cudaEventRecord(ev[b], st), __FILE__, __LINE__))) break;
  }
  if (!rc) rc = cuda_rc(cudaStreamSynchronize(st), __FILE__, __LINE__);
  cleanup();
  if (rc) {
    for (int i = 0; i < n; ++i) {
      qweight_destroy(out[i]);
      out[i] = nullptr;
    }
    return rc;
  }
  if (bytes) *bytes = total;
  return N730_OK;
}

}  // namespace n730

using namespace n730;

N730_API int n730_qweight_load_blocks(const char* path, int n, const int64_t* offsets, void* stream,
                                      void** out_handles, int64_t* bytes_read) {
  return load_blocks(path, n, offsets, (cudaStream_t)stream, reinterpret_cast<QWeight**>(out_handles), bytes_read);
}
