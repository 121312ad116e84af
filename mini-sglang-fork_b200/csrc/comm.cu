// Kernel 3 (tensor-parallel communicator) — placeholder until the peer-memory
// reduce lands; every entry point reports W8A8_ERR_UNSUPPORTED.
#include "common.cuh"

struct w8a8_comm {
  int rank;
};

extern "C" {

size_t w8a8_comm_handle_bytes(void) { return 0; }

int w8a8_comm_create(int, int, int, size_t, w8a8_comm**, void*) {
  return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet");
}

int w8a8_comm_open_peers(w8a8_comm*, const void*) {
  return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet");
}

int w8a8_comm_set_timeout_ms(w8a8_comm*, int64_t) {
  return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet");
}

int w8a8_all_reduce(w8a8_comm*, void*, int64_t, void*) {
  return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet");
}

int w8a8_gemm_allreduce(w8a8_comm*, const int8_t*, const int8_t*, const float*, const float*, const void*,
                        void*, int64_t, int64_t, int64_t, void*, size_t, void*) {
  return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet");
}

int w8a8_comm_status(w8a8_comm*, int*) { return w8a8::fail(W8A8_ERR_UNSUPPORTED, "comm: not built yet"); }

void w8a8_comm_destroy(w8a8_comm*) {}

}  // extern "C"
