// POSIX stand-ins for the handful of Win32 file-mapping calls that the reference's
// CPU oracle uses (src/cpu_reference.cpp:181-227). TEST INFRASTRUCTURE ONLY.
//
// A HANDLE here is the file descriptor plus one (so fd 0 is never confused with a
// null handle). MapViewOfFile maps the whole file read-only; the reference never
// unmaps before exit in the paths the parity harness uses, so UnmapViewOfFile is a
// no-op (the mapping is released at process exit).
#pragma once
#include <cstddef>
#include <cstdint>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef void* HANDLE;
typedef int BOOL;
typedef unsigned long DWORD;
typedef union {
    long long QuadPart;
} LARGE_INTEGER;

#define INVALID_HANDLE_VALUE ((HANDLE)(intptr_t)-1)
#define GENERIC_READ 0
#define FILE_SHARE_READ 0
#define OPEN_EXISTING 0
#define FILE_ATTRIBUTE_NORMAL 0
#define PAGE_READONLY 0
#define FILE_MAP_READ 0

static inline int g4shim_fd(HANDLE h) { return (int)((intptr_t)h - 1); }

static inline HANDLE CreateFileA(const char* path, int, int, void*, int, int, void*) {
    const int fd = open(path, O_RDONLY);
    return fd < 0 ? INVALID_HANDLE_VALUE : (HANDLE)(intptr_t)(fd + 1);
}

static inline BOOL GetFileSizeEx(HANDLE h, LARGE_INTEGER* size) {
    struct stat st;
    if (fstat(g4shim_fd(h), &st) != 0) return 0;
    size->QuadPart = (long long)st.st_size;
    return 1;
}

// The mapping handle is a dup of the file's descriptor so the reference's destructor can
// close both handles without closing one descriptor twice.
static inline HANDLE CreateFileMappingA(HANDLE h, void*, int, int, int, void*) {
    const int fd = dup(g4shim_fd(h));
    return fd < 0 ? nullptr : (HANDLE)(intptr_t)(fd + 1);
}

static inline void* MapViewOfFile(HANDLE h, int, int, int, size_t) {
    struct stat st;
    const int fd = g4shim_fd(h);
    if (fstat(fd, &st) != 0) return nullptr;
    void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    return p == MAP_FAILED ? nullptr : p;
}

static inline BOOL UnmapViewOfFile(const void*) { return 1; }

static inline BOOL CloseHandle(HANDLE h) {
    if (h && h != INVALID_HANDLE_VALUE) close(g4shim_fd(h));
    return 1;
}
