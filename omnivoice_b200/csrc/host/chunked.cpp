// ChunkedSynthesis (chunked.hpp): chunk 0, then the remaining chunks spread
// over the generators, one host thread and one packed batch per GPU.
#include "chunked.hpp"

#include <algorithm>
#include <atomic>
#include <exception>
#include <mutex>
#include <thread>
#include <utility>

namespace gufo::models::omnivoice {
namespace {

void SetError(std::string* error, std::string message) {
  if (error != nullptr) *error = std::move(message);
}

// Longest-processing-time-first assignment of chunks to `workers` by their
// packed rows (the hot path's work grows with them); ties by index.
std::vector<std::vector<std::size_t>> Partition(const std::vector<std::size_t>& indices,
                                                const std::vector<std::size_t>& rows,
                                                std::size_t workers) {
  std::vector<std::size_t> order(indices.size());
  for (std::size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](std::size_t a, std::size_t b) { return rows[a] > rows[b]; });
  std::vector<std::vector<std::size_t>> parts(workers);
  std::vector<std::size_t> load(workers, 0);
  for (const std::size_t k : order) {
    const std::size_t w =
        static_cast<std::size_t>(std::min_element(load.begin(), load.end()) - load.begin());
    parts[w].push_back(indices[k]);
    load[w] += rows[k];
  }
  for (auto& p : parts) std::sort(p.begin(), p.end());
  return parts;
}

}  // namespace

ChunkedSynthesis::ChunkedSynthesis(std::vector<Generator*> generators, std::vector<Codec*> codecs)
    : generators_(std::move(generators)), codecs_(std::move(codecs)) {}

bool ChunkedSynthesis::Run(std::size_t count, const BuildInput& build, bool has_reference,
                           const DecodingConfig& decoding, std::uint64_t seed,
                           const std::function<bool()>& cancelled,
                           std::vector<SynthesizedChunk>* chunks, std::string* error) {
  if (chunks == nullptr || count == 0 || generators_.empty()) {
    SetError(error, "OmniVoice synthesis: no chunks or no generator");
    return false;
  }
  if (!codecs_.empty() && codecs_.size() != generators_.size()) {
    SetError(error, "OmniVoice synthesis: one codec per generator");
    return false;
  }
  chunks->assign(count, SynthesizedChunk{});
  // Decodes chunk i with GPU g's codec (when there is one).
  auto decode = [&](std::size_t g, std::size_t i, std::string* err) {
    if (codecs_.empty()) return true;
    SynthesizedChunk& c = (*chunks)[i];
    return codecs_[g]->Decode(c.codes, c.frames, &c.audio, err);
  };

  CarriedVoice voice;
  const CarriedVoice* carried = nullptr;
  std::size_t first = 0;
  if (!has_reference && count > 1) {
    ConditionalInput input;
    GenerationResult result;
    if (!build(0, nullptr, &input, error)) return false;
    if (!generators_[0]->Generate(input, decoding, seed, cancelled, &result, error)) return false;
    SynthesizedChunk& c = (*chunks)[0];
    c.frames = input.target_frames;
    c.codes = std::move(result.codes);
    if (!decode(0, 0, error)) return false;
    voice.index = 0;
    voice.codes = c.codes;
    voice.frames = c.frames;
    carried = &voice;
    first = 1;
  }

  // The remaining chunks: their inputs, then one packed batch per GPU.
  std::vector<std::size_t> rest;
  std::vector<ConditionalInput> inputs(count);
  std::vector<std::size_t> rows;
  for (std::size_t i = first; i < count; ++i) {
    if (!build(i, carried, &inputs[i], error)) return false;
    rest.push_back(i);
    rows.push_back(inputs[i].length + inputs[i].target_frames);
  }
  const std::size_t workers = std::min(generators_.size(), rest.size());
  const auto parts = Partition(rest, rows, workers);
  std::mutex failure_mutex;
  std::string failure;
  std::atomic<bool> failed{false};
  const auto stop = [&] { return failed.load() || (cancelled && cancelled()); };
  auto work = [&](std::size_t g) {
    std::string err;
    bool ok = true;
    try {
      std::vector<ConditionalInput> batch;
      for (const std::size_t i : parts[g]) batch.push_back(inputs[i]);
      std::vector<std::uint64_t> seeds(batch.size(), seed);
      std::vector<GenerationResult> results;
      ok = generators_[g]->GenerateBatch(batch, decoding, seeds, stop, &results, &err);
      for (std::size_t k = 0; ok && k < parts[g].size(); ++k) {
        SynthesizedChunk& c = (*chunks)[parts[g][k]];
        c.frames = batch[k].target_frames;
        c.codes = std::move(results[k].codes);
        ok = decode(g, parts[g][k], &err);
      }
    } catch (const std::exception& e) {
      ok = false;
      err = std::string("OmniVoice synthesis: ") + e.what();
    }
    if (!ok) {
      std::lock_guard<std::mutex> lock(failure_mutex);
      // The first failure is the cause; the others were stopped by it.
      if (!failed.exchange(true)) failure = err;
    }
  };
  if (workers == 1) {
    work(0);
  } else if (workers > 1) {
    std::vector<std::thread> threads;
    for (std::size_t g = 0; g < workers; ++g) threads.emplace_back(work, g);
    for (auto& t : threads) t.join();
  }
  if (failed.load()) {
    SetError(error, failure);
    return false;
  }
  return true;
}

}  // namespace gufo::models::omnivoice
