#include "Tokens.h"

#include <algorithm>
#include <fstream>
#include <stdexcept>

xt::xtensor<uint32_t, 1> read_tokens(std::istream& input) {
    std::vector<uint32_t> ids;
    unsigned char b[4];
    while (input.read(reinterpret_cast<char*>(b), 4))
        ids.push_back(uint32_t(b[0]) | (uint32_t(b[1]) << 8) | (uint32_t(b[2]) << 16) | (uint32_t(b[3]) << 24));
    xt::xtensor<uint32_t, 1> out = xt::empty<uint32_t>({ids.size()});
    std::copy(ids.begin(), ids.end(), out.data());
    return out;
}

uint32_t pad_token_id(const std::string& vocab_file) {
    std::ifstream f(vocab_file);
    if (!f) throw std::runtime_error("cannot open " + vocab_file);
    std::string line;
    while (std::getline(f, line)) {
        const auto tab = line.find('\t');
        if (tab == std::string::npos) continue;
        if (line.compare(tab + 1, std::string::npos, "<|pad|>") == 0)
            return static_cast<uint32_t>(std::stoul(line.substr(0, tab)));
    }
    return 0;
}

xt::xtensor<uint32_t, 2> token_batch(const std::vector<std::string>& files, uint32_t pad) {
    std::vector<xt::xtensor<uint32_t, 1>> seqs;
    std::size_t max_len = 0;
    for (const auto& path : files) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("Cannot open file: " + path);
        seqs.push_back(read_tokens(f));
        max_len = std::max(max_len, seqs.back().size());
    }
    xt::xtensor<uint32_t, 2> batch = xt::empty<uint32_t>({seqs.size(), max_len});
    for (std::size_t i = 0; i < seqs.size(); ++i) {
        uint32_t* row = batch.data() + i * max_len;
        std::copy(seqs[i].data(), seqs[i].data() + seqs[i].size(), row);
        std::fill(row + seqs[i].size(), row + max_len, pad);
    }
    return batch;
}
