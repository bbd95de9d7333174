/*
 * mb200_peer.h — C ABI of the NVLink peer-memory exchange of the multi-GPU SpMV.
 *
 * The reference's cusparseSpMV (libraries/sparse/src/cusparse_ops.mm:71-211) is a
 * single-device call; across GPUs the row-block product has one exchange step, the
 * vector x.  This library replaces the all-gather before the local product: every
 * rank pulls the other ranks' x blocks straight from their HBM over NVLink /
 * NVSwitch (16-byte loads of peer memory mapped by CUDA IPC), with per-epoch flags
 * instead of a collective.  There is no reference interface for it; the caller is
 * muda_b200/dist_spmv.py.
 *
 * Exchange buffer of one rank (mb200PeerAlloc): a 256-byte header, then two x
 * buffers of `count` floats.  Header word p (p < MB200_PEER_MAX_RANKS) holds the
 * last epoch rank p announced to this rank; word MB200_PEER_STATUS_WORD collects
 * bit p when a wait for rank p ran out.  Epoch e uses x buffer e % 2, so a rank can
 * fill the next epoch's block while peers still read the current one (a peer
 * announces epoch e + 1 only after its own pull of epoch e has finished).
 */
#ifndef MUDA_B200_PEER_H_
#define MUDA_B200_PEER_H_

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MB200_PEER_SUCCESS = 0,
  MB200_PEER_INVALID_VALUE = 1,
  MB200_PEER_CUDA_ERROR = 2
} mb200PeerStatus_t;

#define MB200_PEER_HANDLE_BYTES 64
#define MB200_PEER_MAX_RANKS 32
#define MB200_PEER_STATUS_WORD 48

/* Allocates and zeroes this rank's exchange buffer for `count` floats per x buffer
 * on the current device and writes its IPC handle (MB200_PEER_HANDLE_BYTES bytes). */
mb200PeerStatus_t mb200PeerAlloc(size_t count, void** base, void* handle);

/* Maps another rank's exchange buffer from its IPC handle. */
mb200PeerStatus_t mb200PeerOpen(const void* handle, void** peer_base);

/* Unmaps a buffer opened by mb200PeerOpen. */
mb200PeerStatus_t mb200PeerClose(void* peer_base);

/* Frees this rank's buffer (after every peer has closed it). */
mb200PeerStatus_t mb200PeerFree(void* base);

/* The x buffer that epoch `epoch` uses inside an exchange buffer. */
float* mb200PeerBuffer(void* base, size_t count, unsigned epoch);

/* Epoch `epoch` (1, 2, ... in order) on `stream`: copies x_local (`block` floats)
 * to offset rank * block of this rank's epoch buffer, announces the epoch to every
 * peer, then for each peer waits (at most about one second) for its announcement
 * and pulls its block into the same offsets of this rank's buffer.  bases[p] is
 * rank p's exchange buffer as mapped here (this rank's own at bases[rank]);
 * world * block <= count.  A wait that runs out sets bit p of the status word and
 * skips that block, so the call always completes; while the bit stays set (until
 * mb200PeerTakeStatus), later calls skip peer p without waiting. */
mb200PeerStatus_t mb200PeerAllgather(void* const* bases, int world, int rank, size_t count,
                                     size_t block, unsigned epoch, const float* x_local,
                                     cudaStream_t stream);

/* Reads (after synchronising the device) and clears this rank's status word. */
mb200PeerStatus_t mb200PeerTakeStatus(void* base, unsigned* status);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_PEER_H_ */
