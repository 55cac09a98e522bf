/* blockscan_oracle.c -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 * Mamba-3 block scan (Scan-B) restatement; filled in with the block path. */
#include "oracle.h"
