// Device table of a peer-to-peer all-reduce group (see p2p.cu).
#pragma once

#include <stdint.h>

namespace tllm {

constexpr int kP2PMaxRanks = 8;

struct P2PDev {
  int rank, size, mmax, ncols;
  float *recv_local;                   // [2][size][mmax][ncols]
  int *flags_local;                    // [size]
  int *state;                          // {epoch, ticket} (this rank only)
  float *peer_recv[kP2PMaxRanks];      // every rank's recv (own included)
  int *peer_flags[kP2PMaxRanks];       // every rank's flags (own included)
};

// The device table of a context from tllm_p2p_create after checking that
// rows x cols fit its receive slots; NULL (with the error string set) if not.
const P2PDev *p2p_table(const void *ctx, int rows, int cols);

}  // namespace tllm
