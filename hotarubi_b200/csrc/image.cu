// Weights straight from a compiled program (include/hrb_gemm.h section 9).
//
// hotarubi's compiler writes one DDR image per model, image.bin, and a
// meta.json whose "regions" object maps every named allocation to
// [offset, size] in it (MetaJson, tools/compiler/output.cpp:57-62; read back
// by LoadProgram, include/hotarubi/runtime.hpp:44-56).  A Linear's weights
// are a region of WBUF words as PackWbuf lays them out (tools/compiler/
// tensors.cpp:66-90): an MXFP4 matrix as one region, a W8 matrix as two,
// "<name>_hi" and "<name>_lo" (PlaceW8, tools/compiler/smolvla_common.cpp:
// 95-103).  Here the image is uploaded once; a region becomes dense weights
// on the device (the WBUF translators) the first time a GEMM names it, and
// stays cached in the image for the GEMMs after.
#include <cuda_runtime.h>

#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "hrb_gemm.h"
#include "hrb_kernels.cuh"

struct hrb_image {
  hrb_ctx* ctx = nullptr;
  uint8_t* d_bytes = nullptr;
  size_t bytes = 0;
  // Regions already turned into dense weights [N][kp(/2)] + scales [N][kb].
  struct Dense {
    uint32_t wfmt;
    uint64_t offset, offset_lo;
    uint32_t n, kb;
    uint8_t* w;
    uint8_t* ws;
  };
  std::vector<Dense> dense;
  std::mutex mu;
};

namespace {

constexpr uint64_t kWordBytes = 144;  // one WBUF word in DDR

hrb_status fail(hrb_ctx* ctx, hrb_status st, const char* msg) { return hrb::ctx_fail(ctx, st, msg); }

// JSON scanning for the compiler's meta.json (MetaJson writes it compact; any
// whitespace is skipped).
const char* skip_ws(const char* p) {
  while (*p != '\0' && std::isspace(static_cast<unsigned char>(*p))) ++p;
  return p;
}

// Past the JSON value at p (string, number, literal, array or object), or
// nullptr when it is malformed.
const char* skip_value(const char* p) {
  p = skip_ws(p);
  if (*p == '"') {
    for (++p; *p != '\0' && *p != '"'; ++p) {
      if (*p == '\\' && p[1] != '\0') ++p;
    }
    return *p == '"' ? p + 1 : nullptr;
  }
  if (*p == '[' || *p == '{') {
    const char close = *p == '[' ? ']' : '}';
    p = skip_ws(p + 1);
    if (*p == close) return p + 1;
    while (true) {
      if (close == '}') {
        p = skip_value(p);  // the key
        if (p == nullptr) return nullptr;
        p = skip_ws(p);
        if (*p != ':') return nullptr;
        ++p;
      }
      p = skip_value(p);
      if (p == nullptr) return nullptr;
      p = skip_ws(p);
      if (*p == ',') {
        ++p;
        continue;
      }
      return *p == close ? p + 1 : nullptr;
    }
  }
  const char* q = p;
  while (*q != '\0' && *q != ',' && *q != ']' && *q != '}' &&
         !std::isspace(static_cast<unsigned char>(*q))) {
    ++q;
  }
  return q == p ? nullptr : q;
}

// Inside the object whose '{' is at p: the value of member `key`, or nullptr.
const char* find_member(const char* p, const char* key) {
  p = skip_ws(p);
  if (*p != '{') return nullptr;
  p = skip_ws(p + 1);
  const size_t klen = std::strlen(key);
  while (*p == '"') {
    const char* name = p + 1;
    const char* after = skip_value(p);
    if (after == nullptr) return nullptr;
    const bool match = static_cast<size_t>(after - 1 - name) == klen &&
                       std::strncmp(name, key, klen) == 0;
    p = skip_ws(after);
    if (*p != ':') return nullptr;
    p = skip_ws(p + 1);
    if (match) return p;
    p = skip_value(p);
    if (p == nullptr) return nullptr;
    p = skip_ws(p);
    if (*p != ',') return nullptr;
    p = skip_ws(p + 1);
  }
  return nullptr;
}

bool parse_u64(const char*& p, uint64_t* out) {
  p = skip_ws(p);
  char* end = nullptr;
  const double v = std::strtod(p, &end);  // the writer prints integers as numbers
  if (end == p || v < 0 || v != static_cast<double>(static_cast<uint64_t>(v))) return false;
  *out = static_cast<uint64_t>(v);
  p = end;
  return true;
}

}  // namespace

extern "C" {

hrb_status hrb_image_region(const char* meta_json, const char* name, uint64_t* offset,
                            uint64_t* size) {
  if (meta_json == nullptr || name == nullptr || offset == nullptr || size == nullptr) {
    return HRB_EINVAL;
  }
  const char* regions = find_member(meta_json, "regions");
  if (regions == nullptr) return fail(nullptr, HRB_EINVAL, "meta.json has no regions");
  const char* p = find_member(regions, name);
  if (p == nullptr) {
    std::string msg = std::string("no region ") + name;
    return fail(nullptr, HRB_EINVAL, msg.c_str());
  }
  p = skip_ws(p);
  uint64_t off = 0, sz = 0;
  if (*p != '[' || !parse_u64(++p, &off)) return fail(nullptr, HRB_EINVAL, "bad region entry");
  p = skip_ws(p);
  if (*p != ',' || !parse_u64(++p, &sz)) return fail(nullptr, HRB_EINVAL, "bad region entry");
  p = skip_ws(p);
  if (*p != ']') return fail(nullptr, HRB_EINVAL, "bad region entry");
  *offset = off;
  *size = sz;
  return HRB_OK;
}

hrb_status hrb_image_upload(hrb_ctx* ctx, const void* bytes, size_t n, hrb_image** out) {
  if (ctx == nullptr || bytes == nullptr || n == 0 || out == nullptr) return HRB_EINVAL;
  *out = nullptr;
  if (cudaSetDevice(hrb::ctx_device(ctx)) != cudaSuccess) {
    return fail(ctx, HRB_ECUDA, "cudaSetDevice");
  }
  auto* img = new (std::nothrow) hrb_image;
  if (img == nullptr) return fail(ctx, HRB_ENOMEM, "image");
  img->ctx = ctx;
  img->bytes = n;
  if (cudaMalloc(&img->d_bytes, n) != cudaSuccess) {
    delete img;
    return fail(ctx, HRB_ENOMEM, "image upload: cudaMalloc");
  }
  if (cudaMemcpy(img->d_bytes, bytes, n, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(img->d_bytes);
    delete img;
    return fail(ctx, HRB_ECUDA, "image upload: cudaMemcpy");
  }
  *out = img;
  return HRB_OK;
}

hrb_status hrb_image_destroy(hrb_image* image) {
  if (image == nullptr) return HRB_OK;
  cudaSetDevice(hrb::ctx_device(image->ctx));
  cudaStreamSynchronize(static_cast<cudaStream_t>(hrb_get_stream(image->ctx)));
  for (auto& d : image->dense) {
    cudaFree(d.w);
    cudaFree(d.ws);
  }
  cudaFree(image->d_bytes);
  delete image;
  return HRB_OK;
}

const void* hrb_image_data(const hrb_image* image) {
  return image == nullptr ? nullptr : image->d_bytes;
}

hrb_status hrb_image_weights(hrb_ctx* ctx, const hrb_image* image, uint32_t wfmt,
                             uint64_t offset, uint64_t offset_lo, uint32_t N, uint32_t K,
                             uint8_t* w, uint8_t* wscale, void* stream) {
  if (ctx == nullptr || image == nullptr || w == nullptr || wscale == nullptr) return HRB_EINVAL;
  if (wfmt == HRB_WFMT_MXFP8) {
    return fail(ctx, HRB_ENOTSUP, "the compiler places no MXFP8 weights (no WBUF format)");
  }
  if (wfmt > HRB_WFMT_MXFP8 || N == 0 || N % 8 != 0 || K == 0 || K % 32 != 0) {
    return fail(ctx, HRB_EINVAL, "image weights: N a multiple of 8, K of 32");
  }
  const uint32_t groups = N / 8, kb = K / 32;
  const uint64_t plane = uint64_t{groups} * kb * kWordBytes;
  const uint64_t first = offset, second = wfmt == HRB_WFMT_W8 ? offset_lo : offset;
  if (first + plane > image->bytes || second + plane > image->bytes) {
    return fail(ctx, HRB_EINVAL, "weight region past the end of the image");
  }
  if (wfmt == HRB_WFMT_MXFP4) {
    return hrb_wbuf_to_dense(ctx, image->d_bytes + first, groups, kb, w, wscale, stream);
  }
  return hrb_w8_planes_to_dense(ctx, image->d_bytes + first, image->d_bytes + second, groups,
                                kb, reinterpret_cast<int8_t*>(w), wscale, stream);
}

hrb_status hrb_gemm_image(hrb_ctx* ctx, hrb_image* image, const hrb_gemm_desc* desc,
                          uint64_t offset, uint64_t offset_lo, void* stream) {
  if (ctx == nullptr || image == nullptr || desc == nullptr) return HRB_EINVAL;
  if (desc->w != nullptr || desc->wscale != nullptr) {
    return fail(ctx, HRB_EINVAL, "hrb_gemm_image takes its weights from the image: w = NULL");
  }
  const uint32_t kb = (desc->K + 31u) / 32u, kp = kb * 32u;
  // The region holds whole groups of 8 columns (the compiler pads rows).
  const uint32_t n8 = (desc->N + 7u) / 8u * 8u;
  hrb_image::Dense use{};
  {
    std::lock_guard<std::mutex> lock(image->mu);
    bool have = false;
    for (const auto& d : image->dense) {
      if (!have && d.wfmt == desc->wfmt && d.offset == offset &&
          (desc->wfmt != HRB_WFMT_W8 || d.offset_lo == offset_lo) && d.n == n8 && d.kb == kb) {
        use = d;
        have = true;
      }
    }
    if (!have) {
      hrb_image::Dense d{desc->wfmt, offset, offset_lo, n8, kb, nullptr, nullptr};
      const size_t wbytes = static_cast<size_t>(n8) * (desc->wfmt == HRB_WFMT_MXFP4 ? kp / 2 : kp);
      if (cudaSetDevice(hrb::ctx_device(ctx)) != cudaSuccess ||
          cudaMalloc(&d.w, wbytes) != cudaSuccess ||
          cudaMalloc(&d.ws, static_cast<size_t>(n8) * kb) != cudaSuccess) {
        cudaFree(d.w);
        return fail(ctx, HRB_ENOMEM, "image weights: cudaMalloc");
      }
      const hrb_status st =
          hrb_image_weights(ctx, image, desc->wfmt, offset, offset_lo, n8, kp, d.w, d.ws, stream);
      if (st != HRB_OK) {
        cudaFree(d.w);
        cudaFree(d.ws);
        return st;
      }
      image->dense.push_back(d);
      use = d;
    }
  }
  hrb_gemm_desc g = *desc;
  g.w = use.w;
  g.wscale = use.ws;
  return hrb_gemm_dense(ctx, &g, stream);
}

}  // extern "C"
