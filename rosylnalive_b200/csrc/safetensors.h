// safetensors.h -- the safetensors header model and validator (internal; the C ABI is lrm_st_* in lrm_cuda.h).
#pragma once

#include <stdint.h>

#include <string>
#include <utility>
#include <vector>

namespace lrm {
namespace st {

// dtype codes: the order of LRM_ST_* (F32, F64, BF16, F16, I32, U32, U8, I64).
struct Entry {
    std::string name;
    int dtype = -1;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte offsets within the data section
};

struct Parsed {
    uint64_t header_len = 0;
    std::vector<Entry> entries;                                 // code point order of the names
    std::vector<std::pair<std::string, std::string>> metadata;  // code point order of the keys
};

// Validates a whole file image (8-byte length, header, data) and fills `out`; throws st::FormatError (defined in
// safetensors.cpp) with the reason.
void parse(const uint8_t *bytes, uint64_t length, Parsed &out);

int dtype_size(int dtype);

}  // namespace st
}  // namespace lrm
