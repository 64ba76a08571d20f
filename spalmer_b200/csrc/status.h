// Status codes: the public ones come from include/spx.h; the device-side
// status word values below are reported through spx_workspace_status.
#pragma once

#include "../../include/spx.h"

#define SPX_DEV_TIMEOUT_PRODUCER 0x101
#define SPX_DEV_TIMEOUT_MMA 0x102
#define SPX_DEV_TIMEOUT_EPILOGUE 0x103
#define SPX_DEV_BAD_EXPERT 0x201
#define SPX_DEV_BAD_TILE 0x202
