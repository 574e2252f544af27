// OLMo-2-0425-1B shape constants under the names the reference uses
// (model_config.h:3-7 of the DirkTensor tree), so code written against them
// compiles unchanged with the drop-in.
#pragma once

static constexpr unsigned int head_dim = 128;
static constexpr unsigned int max_seq_len = 8192;
static constexpr unsigned int d_model = 2048;
static constexpr unsigned int n_heads = d_model / head_dim;
static constexpr unsigned int n_layers = 16;
