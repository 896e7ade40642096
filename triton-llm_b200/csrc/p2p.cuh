// Device table of a peer-to-peer all-reduce group (see p2p.cu).
#pragma once

#include <stdint.h>

namespace tllm {

constexpr int kP2PMaxRanks = 8;

// One received value: the fp32 bits in the low half, the number of the call
// that wrote it in the high half, stored and loaded as one 64-bit word.
__host__ __device__ inline unsigned long long p2p_word(float v, unsigned epoch) {
  union {
    float f;
    unsigned u;
  } c;
  c.f = v;
  return ((unsigned long long)epoch << 32) | c.u;
}

struct P2PDev {
  int rank, size, mmax, ncols;
  unsigned long long *recv_local;                 // [2][size][mmax][ncols]
  int *state;                                     // {calls done, reader ticket}
  unsigned long long *peer_recv[kP2PMaxRanks];    // every rank's recv (own too)
};

// The device table of a context from tllm_p2p_create after checking that
// rows x cols fit its receive slots; NULL (with the error string set) if not.
const P2PDev *p2p_table(const void *ctx, int rows, int cols);

}  // namespace tllm
