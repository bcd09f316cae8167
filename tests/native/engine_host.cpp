// Host build of the engine headers, for the CPU parity tests only.
//
// The product runs these headers inside CUDA kernels (cugo_b200/csrc/); this
// file compiles the very same rule code with g++ so that the CPU test suite can
// compare it against the oracle row by row without a GPU.  Nothing in the
// package loads this library.
#include <cstdint>
#include <cstring>

#include "../../cugo_b200/csrc/engine/driver.cuh"
#include "../../cugo_b200/csrc/engine/env.cuh"

using namespace cb;

namespace {
Game load(const uint8_t* row) {
  Game g;
  std::memcpy(g.w, row, kRowBytes);
  return g;
}
void save(Game g, uint8_t* row) {
  zero_padding(g);
  std::memcpy(row, g.w, kRowBytes);
}
}  // namespace

extern "C" {

void cugo_host_create(const int64_t* seeds, const int64_t* first, int64_t n, uint8_t* rows) {
  for (int64_t i = 0; i < n; ++i) {
    Game g;
    create_game(g, static_cast<u64>(seeds[i]), static_cast<u32>(first[i] & 1));
    save(g, rows + i * kRowBytes);
  }
}

void cugo_host_observe(const uint8_t* rows, int64_t n, float* features, uint8_t* legal,
                       uint8_t* player, uint8_t* done, int16_t* status) {
  for (int64_t i = 0; i < n; ++i) {
    const Game g = load(rows + i * kRowBytes);
    ObsPacket pk;
    ObsMeta meta;
    observe_game(g, pk.ref(), meta);
    for (u32 c = 0; c < kFeatures; ++c) features[i * kFeatures + c] = feature_value(pk, c);
    for (u32 a = 0; a < kActions; ++a) legal[i * kActions + a] = meta.legal.has(a) ? 1 : 0;
    player[i] = static_cast<uint8_t>(meta.player);
    done[i] = static_cast<uint8_t>(meta.done);
    status[i] = static_cast<int16_t>(meta.status);
  }
}

void cugo_host_step(uint8_t* rows, const int64_t* actions, int64_t n, float* reward,
                    uint8_t* done, uint8_t* nagari, int16_t* status, uint8_t* committed,
                    int64_t* events) {
  for (int64_t i = 0; i < n; ++i) {
    Game g = load(rows + i * kRowBytes);
    const EventBase base = event_base(g);
    const int64_t raw = actions[i];
    const u32 action = raw >= 0 && raw < kActions ? static_cast<u32>(raw) : kNoAction;
    const StepOut r = step_game(g, action);
    reward[i] = static_cast<float>(r.reward0);
    done[i] = static_cast<uint8_t>(r.done);
    nagari[i] = static_cast<uint8_t>(r.nagari);
    status[i] = static_cast<int16_t>(r.status);
    committed[i] = static_cast<uint8_t>(r.committed);
    if (events != nullptr) {
      if (r.committed) event_words(base, g, events + i * kEventWords);
      else std::memset(events + i * kEventWords, 0, kEventWords * sizeof(int64_t));
    }
    save(g, rows + i * kRowBytes);
  }
}

void cugo_host_start(const uint8_t* rows, int64_t n, int64_t* out) {
  for (int64_t i = 0; i < n; ++i) start_words(load(rows + i * kRowBytes), out + i * kStartWords);
}

void cugo_host_stock(const uint8_t* rows, int64_t n, int64_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = static_cast<int64_t>(stock_preview(load(rows + i * kRowBytes)));
}

uint32_t cugo_host_philox_word(uint64_t game, uint32_t decision, uint32_t stream, uint64_t seed) {
  return game_draw(game, decision, stream, seed).v[0];
}

void cugo_host_philox(const uint32_t* ctr, const uint32_t* key, uint32_t* out) {
  const Philox4 p = philox4x32_10(ctr[0], ctr[1], ctr[2], ctr[3], key[0], key[1]);
  for (int i = 0; i < 4; ++i) out[i] = p.v[i];
}

// Rows at which primary_action_legal disagrees with the primary legal mask (every
// action 0..255 of every row); mismatches[i] = the first such action or -1.
void cugo_host_legal_check(const uint8_t* rows, int64_t n, int32_t* mismatches) {
  for (int64_t i = 0; i < n; ++i) {
    const Game g = load(rows + i * kRowBytes);
    const Legal m = primary_legal(g);
    mismatches[i] = -1;
    for (uint32_t a = 0; a < 256; ++a) {
      if (m.has(a) != primary_action_legal(g, a)) {
        mismatches[i] = static_cast<int32_t>(a);
        break;
      }
    }
  }
}

}  // extern "C"
