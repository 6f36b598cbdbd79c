// TEST INFRASTRUCTURE — POSIX stand-ins for the two MSVC C runtime calls the reference's
// bench source uses (localtime_s with the MSVC argument order, _fseeki64), so that it compiles
// with gcc under nvcc. Nothing else of the bench is changed.
#pragma once
#include <cstdio>
#include <ctime>
#include <sys/types.h>

static inline int localtime_s(struct tm* sortie, const time_t* t) { return localtime_r(t, sortie) ? 0 : 1; }
static inline int _fseeki64(FILE* f, long long decalage, int origine) { return fseeko(f, (off_t)decalage, origine); }
