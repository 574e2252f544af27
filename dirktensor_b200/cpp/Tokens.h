// Token input of the driver (main.cpp:14-58): the uint32 token-file reader,
// the pad-token lookup in vocab.txt (Detokenizer.cpp:41-80) and the padded
// batch main() builds from several token files.  Host-side byte work; it feeds
// OlmoModel::forward.
#pragma once

#include <cstdint>
#include <istream>
#include <string>
#include <vector>

#include <xtensor/containers/xtensor.hpp>

// Reads little-endian uint32 token ids until EOF (main.cpp:14-27).  A trailing
// partial id (file size not a multiple of 4) is ignored, as the reference's
// read loop ignores it.
xt::xtensor<uint32_t, 1> read_tokens(std::istream& input);

// The id of "<|pad|>" in a vocab.txt of "id<TAB>token" lines (0 when absent, the
// reference's default).  Throws std::runtime_error when the file cannot be opened.
uint32_t pad_token_id(const std::string& vocab_file);

// One row per token file, right-padded with `pad` to the longest file
// (main.cpp:33-58).  Throws std::runtime_error when a file cannot be opened.
xt::xtensor<uint32_t, 2> token_batch(const std::vector<std::string>& files, uint32_t pad);
