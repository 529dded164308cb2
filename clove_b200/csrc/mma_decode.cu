#include "mma_decode.cuh"
