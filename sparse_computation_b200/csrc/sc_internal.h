// Internal types shared by the host (formats, coarsening) and device (plan,
// kernels) halves of libsc_b200.so.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "sc_b200.h"

struct sc_error : std::runtime_error {
  int code;
  sc_error(int c, const std::string &msg) : std::runtime_error(msg), code(c) {}
};

// CSR with int32 indices and float64 values, like sym_lib::CSR
// (aggregation/include/aggregation/def.h:181) and scipy's csr_matrix.
struct sc_csr {
  int32_t m = 0, n = 0;
  std::vector<int32_t> rowptr, colind;
  std::vector<double> vals;
};

// One pattern block of a CF matrix (CompressedFormat<T>,
// include/compressed_format/CompressedFormat.h:88-221): RPP has one entry per
// row panel plus one; CB holds the padded column list; the values of column
// CB[j] for the pattern's rows are vals[j*popcount .. j*popcount+popcount).
struct sc_pattern {
  std::string mask;   // '1'/'0' per panel row, panel row 0 first
  int32_t popcount = 0;
  std::vector<int32_t> rpp, cb;
  std::vector<float> vals;     // float32, as the reference's loader holds them
  std::vector<double> vals_d;  // float64 source values (for byte-exact writing)
  std::vector<uint8_t> pad;    // 1 where the value token is coarsening padding
  // Raw value tokens when loaded from text and written back unchanged.
  std::vector<std::string> tokens;
};

struct sc_cf {
  int32_t num_rows = 0, num_cols = 0, kernel_m = 0;
  int32_t vector_length_hdr = 0;  // header's 5th field exactly as written/read
  // Header lines "<mask> <id> " in file order (dictionary insertion order).
  std::vector<std::pair<std::string, int32_t>> header;
  std::vector<sc_pattern> pats;   // body order (pattern id order)
  bool from_text = false;         // loaded by sc_cf_load (tokens kept)
  int64_t real_nnz = 0;
};

void sc_set_error(const std::string &msg);
void sc_clear_error();

// Python's repr() of a float64 (shortest round-trip digits, repr layout).
std::string sc_py_float_repr(double d);
