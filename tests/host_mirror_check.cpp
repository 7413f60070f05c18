// Builds against the header-only C++ mirror of the reference's operator
// classes and checks, without touching a GPU, that every class compiles and
// that errors reach the caller as sam3::SAM3Error (the reference's
// `throws SAM3Error`). Compiled and run by tests/test_abi.py.
#include <cstdio>

#include "sam3_modules.hpp"

int main() {
  sam3_encoder_config_t cfg;
  if (sam3_config_default(&cfg) != SAM3_OK) return 2;
  int caught = 0;
  sam3::BufferList recycled;
  try {
    sam3::check(nullptr, sam3_sync(nullptr), "sync");
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  sam3_encoder_weights_t w{};
  sam3::ViTEncoder enc(nullptr, w);
  try {
    enc.forward(nullptr, 1, recycled);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  try {
    enc.encodeHost(nullptr, 1, nullptr, nullptr);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  try {
    enc.submitHost(nullptr, 1, nullptr, nullptr);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  try {
    enc.waitHost(1);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  sam3_windowed_encoder_weights_t ww{};
  sam3::SAM3Encoder wenc(nullptr, ww);
  try {
    wenc.forward(nullptr, 1, recycled);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  sam3::LayerNorm ln(nullptr, cfg.embed_dim, nullptr, nullptr, cfg.ln_eps);
  try {
    ln.forward(nullptr, 1, 1, recycled);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG;
  }
  // recycle() empties its list even when the sync before the frees fails
  // (the null context rejects both calls before touching the pointer)
  sam3::BufferList handed_out{reinterpret_cast<void*>(0x1000)};
  try {
    sam3::recycle(nullptr, handed_out);
  } catch (const sam3::SAM3Error& e) {
    caught += e.status == SAM3_ERR_INVALID_ARG && handed_out.empty();
  }
  // fault injection and the wait self-test need a context too
  const bool no_ctx = sam3_set_fault(nullptr, SAM3_FAULT_ALLOC) == SAM3_ERR_INVALID_ARG &&
                      sam3_selftest_wait_timeout(nullptr) == SAM3_ERR_INVALID_ARG &&
                      sam3_get_fault(nullptr) == 0;
  std::printf("caught %d of 8, embed_dim %d, no-context checks %s\n", caught, cfg.embed_dim,
              no_ctx ? "ok" : "failed");
  return caught == 8 && recycled.empty() && no_ctx ? 0 : 1;
}
