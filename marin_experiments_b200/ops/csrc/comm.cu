// Peer-to-peer collectives over NVLink (filled in by the expert-parallel exchange).
#include <cuda_runtime.h>
