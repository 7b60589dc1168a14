// A GPT with `Blocks` decoder blocks: the reference model (include/nn/GPT.h
// in JTPuffer/TempLit) generalised from its fixed four blocks
// (GPT.h:47-50) so the 12-block, d_model 768 data-parallel configuration
// can be built from the same parts: token + position embedding, pre-RMSNorm
// decoder blocks (include/nn/decoder_block.h), a final RMSNorm and the
// vocabulary projection (include/nn/layer.h).  With Blocks == 4 it builds
// the same expression as nn::GPT.
#pragma once

#include "expr/api.h"
#include "nn/attention.h"
#include "nn/decoder_block.h"
#include "nn/embedding.h"
#include "nn/layer.h"

#include <array>
#include <cstdint>
#include <random>
#include <stdexcept>
#include <utility>
#include <vector>

namespace templit_b200 {

template <typename Mat, uint32_t VocabSize, uint32_t MaxSequenceSize, uint32_t EmbeddingSize,
          uint32_t Heads, size_t Blocks>
class DeepGPT {
  using IndexMat = typename Mat::template rebind<uint32_t>;
  using Indices = expr::tensor::NoGradTensor<IndexMat>;
  using Block = nn::DecoderBlock<Mat, EmbeddingSize, Heads>;

  // Row-major [batch, sequence] position ids 0..sequence-1 per row.
  static IndexMat positions_for(uint32_t batch, uint32_t sequence) {
    if (batch == 0 || sequence == 0 || sequence > MaxSequenceSize)
      throw std::invalid_argument("invalid GPT input dimensions");
    IndexMat ids({batch, sequence});
    std::vector<uint32_t> v(static_cast<size_t>(batch) * sequence);
    for (size_t i = 0; i < v.size(); ++i) v[i] = static_cast<uint32_t>(i % sequence);
    ids.set(v);
    return ids;
  }

  template <size_t... I>
  static std::array<Block, Blocks> make_blocks(std::mt19937 &gen, std::index_sequence<I...>) {
    return {((void)I, Block(gen))...};
  }

  template <size_t I, typename X> auto apply_blocks(X &&x) const {
    if constexpr (I == Blocks) {
      return std::forward<X>(x);
    } else {
      return apply_blocks<I + 1>(blocks_[I](std::forward<X>(x), mask_));
    }
  }

  Indices positions_;
  expr::tensor::NoGradTensor<Mat> mask_;
  nn::Embedding<Mat, VocabSize, EmbeddingSize> token_embedding_;
  nn::Embedding<Mat, MaxSequenceSize, EmbeddingSize> position_embedding_;
  std::array<Block, Blocks> blocks_;
  nn::Layer<Mat> projection_;

public:
  DeepGPT(uint32_t batch, uint32_t sequence, std::mt19937 &gen)
      : positions_(positions_for(batch, sequence)),
        mask_(nn::causal_mask<typename Mat::device_type, typename Mat::value_type>(sequence,
                                                                                   sequence)),
        token_embedding_(gen), position_embedding_(gen),
        blocks_(make_blocks(gen, std::make_index_sequence<Blocks>{})),
        projection_(EmbeddingSize, VocabSize, gen) {}

  auto operator()(Indices input) const {
    auto hidden = expr::add(token_embedding_(std::move(input)), position_embedding_(positions_));
    return projection_(expr::rms_norm(apply_blocks<0>(std::move(hidden))));
  }
};

}  // namespace templit_b200
