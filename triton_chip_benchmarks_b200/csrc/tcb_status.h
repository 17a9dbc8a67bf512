// Status codes shared by host entry points and device status words; the
// public definitions live in the C ABI header.
#pragma once
#include "tcb.h"
