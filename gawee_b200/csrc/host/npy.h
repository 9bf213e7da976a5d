// NPY v1/v2 C-order reader and v1 writer, byte-compatible with the reference
// runtime's loadNpy / saveNpy (back/runtime_support.h:138-283): same header
// keys, same 16-byte header padding, dtype tags <f4 <f8 <i4 <i8 (plus |b1 for
// boolean tensors, which the reference runner does not accept).
#pragma once

#include <cstdint>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "ir.h"

namespace gawee {

struct NpyArray {
  DType dtype = DType::F32;
  std::vector<int64_t> shape;
  std::vector<uint8_t> data;
};

inline const char* npy_tag(DType t) {
  switch (t) {
    case DType::F32: return "<f4";
    case DType::F64: return "<f8";
    case DType::I32: return "<i4";
    case DType::I64: return "<i8";
    case DType::I1: return "|b1";
    default: throw std::runtime_error("npy: unsupported dtype");
  }
}

inline DType npy_dtype(const std::string& tag) {
  if (tag == "<f4") return DType::F32;
  if (tag == "<f8") return DType::F64;
  if (tag == "<i4") return DType::I32;
  if (tag == "<i8") return DType::I64;
  if (tag == "|b1" || tag == "<b1" || tag == "|u1") return DType::I1;
  throw std::runtime_error("npy: unsupported dtype tag '" + tag + "'");
}

inline NpyArray npy_load(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("Could not open NPY file: " + path);
  char magic[6];
  in.read(magic, 6);
  if (!in || std::string(magic, 6) != "\x93NUMPY") throw std::runtime_error("Invalid NPY header: " + path);
  char ver[2];
  in.read(ver, 2);
  uint32_t hlen = 0;
  if (ver[0] == 1) {
    uint16_t h;
    in.read(reinterpret_cast<char*>(&h), 2);
    hlen = h;
  } else {
    in.read(reinterpret_cast<char*>(&hlen), 4);
  }
  std::string header(hlen, '\0');
  in.read(&header[0], hlen);
  if (header.find("'fortran_order': False") == std::string::npos)
    throw std::runtime_error("Only C-order NPY arrays are supported: " + path);
  NpyArray a;
  auto dp = header.find("'descr': '");
  if (dp == std::string::npos) throw std::runtime_error("Failed to parse NPY dtype: " + path);
  dp += 10;
  a.dtype = npy_dtype(header.substr(dp, header.find('\'', dp) - dp));
  auto b = header.find('('), e = header.find(')', b);
  if (b == std::string::npos || e == std::string::npos) throw std::runtime_error("Failed to parse NPY shape: " + path);
  std::stringstream ss(header.substr(b + 1, e - b - 1));
  std::string item;
  while (std::getline(ss, item, ',')) {
    size_t s = item.find_first_not_of(" \t");
    if (s == std::string::npos) continue;
    a.shape.push_back(std::stoll(item.substr(s)));
  }
  int64_t n = 1;
  for (auto d : a.shape) n *= d;
  a.data.resize((size_t)n * dtype_size(a.dtype));
  in.read(reinterpret_cast<char*>(a.data.data()), (std::streamsize)a.data.size());
  if (!in) throw std::runtime_error("Truncated NPY payload: " + path);
  return a;
}

inline void npy_save(const std::string& path, DType t, const std::vector<int64_t>& shape, const void* data) {
  std::ofstream out(path, std::ios::binary);
  if (!out) throw std::runtime_error("Could not open output tensor: " + path);
  std::ostringstream sh;
  sh << "(";
  for (size_t i = 0; i < shape.size(); ++i) {
    sh << shape[i];
    if (shape.size() == 1) sh << ",";
    else if (i + 1 != shape.size()) sh << ", ";
  }
  sh << ")";
  std::string header = std::string("{'descr': '") + npy_tag(t) + "', 'fortran_order': False, 'shape': " + sh.str() + ", }";
  while ((10 + header.size() + 1) % 16 != 0) header.push_back(' ');
  header.push_back('\n');
  out.write("\x93NUMPY", 6);
  const char ver[2] = {1, 0};
  out.write(ver, 2);
  uint16_t hl = (uint16_t)header.size();
  out.write(reinterpret_cast<const char*>(&hl), 2);
  out.write(header.data(), (std::streamsize)header.size());
  int64_t n = 1;
  for (auto d : shape) n *= d;
  out.write(static_cast<const char*>(data), (std::streamsize)(n * (int64_t)dtype_size(t)));
}

}  // namespace gawee
