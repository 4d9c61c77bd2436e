// storage.cu -- the reference's VECRSTOR vector file, read straight into GPU
// shards.
//
// Format (crates/vector-index/src/storage/mmap.rs:7-16; writer
// scripts/generate_dataset.py:50-66): a 24-byte header of three little-endian
// u64 -- magic 0x56454352_53544F52 ("VECRSTOR"), number of vectors, dimension
// -- then N x D little-endian f32, row-major. Validation follows
// MmapStorage::open (mmap.rs:171-223): a file shorter than the header or with
// another magic is an invalid header; a file shorter than 24 + N*D*4 bytes is
// a size mismatch; trailing bytes are allowed.
//
// vrs_knn_create_from_file maps the file read-only (sequential read-ahead
// hint) and hands the mapped rows to vrs_knn_create, whose upload copies each
// GPU's row range from the mapping in bounded chunks: no host-side copy of the
// base is made, so a 100M-row file needs no second 38 GB host buffer.
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>

#include "vrs_internal.cuh"

#if defined(__BYTE_ORDER__) && __BYTE_ORDER__ != __ORDER_LITTLE_ENDIAN__
#error "VECRSTOR files are little-endian; this reader assumes a little-endian host"
#endif

namespace {

constexpr uint64_t kMagic = 0x5645435253544F52ull;  // "VECRSTOR" as a big-endian ASCII word
constexpr uint64_t kHeader = 24;

int file_error(const std::string& m) {
  vrs::set_error(VRS_ERR_INVALID_FILE, m);
  return VRS_ERR_INVALID_FILE;
}

// Validated view of one file: either mapped (data != nullptr) or header only.
struct View {
  int fd = -1;
  void* map = nullptr;
  size_t map_len = 0;
  uint64_t n = 0, d = 0;
  const float* data = nullptr;
  ~View() {
    if (map) munmap(map, map_len);
    if (fd >= 0) close(fd);
  }
};

int open_view(const char* path, bool map_rows, View* v) {
  if (!path) return file_error("null path");
  v->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (v->fd < 0) return file_error(std::string(path) + ": " + strerror(errno));
  struct stat st;
  if (fstat(v->fd, &st) != 0) return file_error(std::string(path) + ": " + strerror(errno));
  const uint64_t size = (uint64_t)st.st_size;
  if (size < kHeader)
    return file_error(std::string(path) + ": invalid header: file too small: " + std::to_string(size) +
                      " bytes (minimum 24)");
  uint64_t h[3];
  ssize_t got = pread(v->fd, h, sizeof(h), 0);
  if (got != (ssize_t)sizeof(h)) return file_error(std::string(path) + ": short header read");
  if (h[0] != kMagic) {
    char buf[96];
    snprintf(buf, sizeof(buf), "invalid magic number: 0x%016llX (expected 0x%016llX)",
             (unsigned long long)h[0], (unsigned long long)kMagic);
    return file_error(std::string(path) + ": invalid header: " + buf);
  }
  v->n = h[1];
  v->d = h[2];
  // 24 + n*d*4 without overflow: a header whose data size exceeds 2^64 cannot
  // be backed by any file.
  unsigned __int128 need = (unsigned __int128)v->n * v->d * 4u + kHeader;
  if (need > (unsigned __int128)size)
    return file_error(std::string(path) + ": file size mismatch: expected " +
                      (need >> 64 ? std::string("more than 2^64") : std::to_string((uint64_t)need)) +
                      " bytes, got " + std::to_string(size));
  if (map_rows && v->n * v->d > 0) {
    v->map_len = (size_t)need;
    v->map = mmap(nullptr, v->map_len, PROT_READ, MAP_PRIVATE, v->fd, 0);
    if (v->map == MAP_FAILED) {
      v->map = nullptr;
      return file_error(std::string(path) + ": mmap: " + strerror(errno));
    }
    madvise(v->map, v->map_len, MADV_SEQUENTIAL);
    v->data = reinterpret_cast<const float*>(static_cast<const char*>(v->map) + kHeader);
  }
  return VRS_OK;
}

}  // namespace

extern "C" int vrs_vecrstor_info(const char* path, int64_t* num_vectors, int64_t* dimension) {
  View v;
  int st = open_view(path, false, &v);
  if (st != VRS_OK) return st;
  if (v.n > (uint64_t)INT64_MAX || v.d > (uint64_t)INT64_MAX)
    return file_error(std::string(path) + ": header sizes exceed int64");
  if (num_vectors) *num_vectors = (int64_t)v.n;
  if (dimension) *dimension = (int64_t)v.d;
  return VRS_OK;
}

extern "C" int vrs_vecrstor_write(const char* path, const float* data, int64_t n, int64_t d) {
  if (!path || n < 0 || d < 0 || (n > 0 && d > 0 && !data)) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "vrs_vecrstor_write: bad arguments");
    return VRS_ERR_INVALID_CONFIG;
  }
  FILE* f = fopen(path, "wb");
  if (!f) return file_error(std::string(path) + ": " + strerror(errno));
  const uint64_t h[3] = {kMagic, (uint64_t)n, (uint64_t)d};
  bool ok = fwrite(h, sizeof(h), 1, f) == 1;
  const size_t total = (size_t)n * (size_t)d;
  if (ok && total) ok = fwrite(data, sizeof(float), total, f) == total;
  ok = (fclose(f) == 0) && ok;
  if (!ok) return file_error(std::string(path) + ": write failed: " + strerror(errno));
  return VRS_OK;
}

extern "C" int vrs_knn_create_from_file(const char* path, int32_t num_gpus, int32_t mode,
                                        int32_t metric, vrs_knn** out) {
  if (!out) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "null out");
    return VRS_ERR_INVALID_CONFIG;
  }
  *out = nullptr;
  View v;
  int st = open_view(path, true, &v);
  if (st != VRS_OK) return st;
  if (v.d < 1 || v.d > (uint64_t)INT32_MAX || v.n > (uint64_t)INT64_MAX) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, std::string(path) + ": dimension " + std::to_string(v.d) +
                                               " is outside 1..2^31-1");
    return VRS_ERR_INVALID_CONFIG;
  }
  // The mapping lives until the engine holds its copy on the GPUs.
  return vrs_knn_create(v.data, (int64_t)v.n, (int32_t)v.d, num_gpus, mode, metric, out);
}

// ----------------------------------------------------------------------------
// Standalone centroid file (IvfPqSerializer::save_centroid_file /
// load_centroid_file, crates/vector-index/src/ivf/serializer.rs:255-370): the
// output of k-means training for later IVF builds. Packed little-endian:
// magic u64 0x5652534B4D45414E ("VRSKMEAN"), version u32 = 1, metric u8
// (serializer.rs:397-430, the same codes as vrs_metric), dimension u32, K u32,
// iterations u32, inertia f32, then K x D f32 (29-byte header).
// ----------------------------------------------------------------------------

namespace {
constexpr uint64_t kCentroidMagic = 0x5652534B4D45414Eull;
constexpr uint32_t kCentroidVersion = 1;
constexpr size_t kCentroidHeader = 29;
}  // namespace

extern "C" int vrs_centroid_file_write(const char* path, const float* centroids, int64_t d,
                                       int64_t k, int32_t metric, int64_t iterations,
                                       float inertia) {
  if (!path || d < 0 || k < 0 || iterations < 0 || d > UINT32_MAX || k > UINT32_MAX ||
      iterations > UINT32_MAX || metric < 0 || metric > 9 || (d * k > 0 && !centroids)) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "vrs_centroid_file_write: bad arguments");
    return VRS_ERR_INVALID_CONFIG;
  }
  unsigned char h[kCentroidHeader];
  const uint32_t dd = (uint32_t)d, kk = (uint32_t)k, it = (uint32_t)iterations;
  memcpy(h + 0, &kCentroidMagic, 8);
  memcpy(h + 8, &kCentroidVersion, 4);
  h[12] = (unsigned char)metric;
  memcpy(h + 13, &dd, 4);
  memcpy(h + 17, &kk, 4);
  memcpy(h + 21, &it, 4);
  memcpy(h + 25, &inertia, 4);
  FILE* f = fopen(path, "wb");
  if (!f) return file_error(std::string(path) + ": " + strerror(errno));
  bool ok = fwrite(h, 1, sizeof(h), f) == sizeof(h);
  const size_t total = (size_t)d * (size_t)k;
  if (ok && total) ok = fwrite(centroids, sizeof(float), total, f) == total;
  ok = (fclose(f) == 0) && ok;
  if (!ok) return file_error(std::string(path) + ": write failed: " + strerror(errno));
  return VRS_OK;
}

extern "C" int vrs_centroid_file_read(const char* path, float* out_centroids, int64_t capacity,
                                      int32_t* metric, int64_t* d, int64_t* k, int64_t* iterations,
                                      float* inertia) {
  if (!path) return file_error("null path");
  FILE* f = fopen(path, "rb");
  if (!f) return file_error(std::string(path) + ": " + strerror(errno));
  struct Closer {
    FILE* f;
    ~Closer() { fclose(f); }
  } closer{f};
  unsigned char h[kCentroidHeader];
  const size_t got = fread(h, 1, sizeof(h), f);
  uint64_t magic = 0;
  if (got >= 8) memcpy(&magic, h, 8);
  if (got < 8) return file_error(std::string(path) + ": unexpected end of file");
  if (magic != kCentroidMagic) {
    char buf[96];
    snprintf(buf, sizeof(buf), "expected centroid magic 0x%llX, got 0x%llX",
             (unsigned long long)kCentroidMagic, (unsigned long long)magic);
    return file_error(std::string(path) + ": invalid header: " + buf);
  }
  if (got < 12) return file_error(std::string(path) + ": unexpected end of file");
  uint32_t version;
  memcpy(&version, h + 8, 4);
  if (version != kCentroidVersion)
    return file_error(std::string(path) + ": invalid header: unsupported centroid file version: " +
                      std::to_string(version));
  if (got < 13) return file_error(std::string(path) + ": unexpected end of file");
  if (h[12] > 9)
    return file_error(std::string(path) + ": invalid header: invalid metric code: " + std::to_string(h[12]));
  if (got < sizeof(h)) return file_error(std::string(path) + ": unexpected end of file");
  uint32_t dd, kk, it;
  float in;
  memcpy(&dd, h + 13, 4);
  memcpy(&kk, h + 17, 4);
  memcpy(&it, h + 21, 4);
  memcpy(&in, h + 25, 4);
  const uint64_t total = (uint64_t)dd * kk;
  if (out_centroids) {
    if ((uint64_t)capacity < total) {
      vrs::set_error(VRS_ERR_INVALID_CONFIG, "vrs_centroid_file_read: capacity " + std::to_string(capacity) +
                                                 " < K x D = " + std::to_string(total));
      return VRS_ERR_INVALID_CONFIG;
    }
    if (total && fread(out_centroids, sizeof(float), (size_t)total, f) != total)
      return file_error(std::string(path) + ": unexpected end of file");
  }
  if (metric) *metric = h[12];
  if (d) *d = dd;
  if (k) *k = kk;
  if (iterations) *iterations = it;
  if (inertia) *inertia = in;
  return VRS_OK;
}
