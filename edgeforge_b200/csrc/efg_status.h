/* efg_status.h - status codes for internal code: the public ones of include/efg.h. */
#ifndef EFG_STATUS_H
#define EFG_STATUS_H
#include "../../include/efg.h"
#endif
