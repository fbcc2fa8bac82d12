/*
 * TEST INFRASTRUCTURE ONLY. A POSIX stand-in for the nine Win32 file calls the reference's
 * src/cpu_reference.cpp makes (:167-219 and :269-282), so that file compiles and runs on
 * Linux unmodified for the oracle/_ref build. Only the semantics that file relies on are
 * provided: open for read, size, map read-only, seek, read, close.
 */
#pragma once
#include <cstdint>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef void* HANDLE;
typedef uint32_t DWORD;
typedef int BOOL;
typedef long long LONGLONG;
typedef union { struct { uint32_t LowPart; int32_t HighPart; } u; LONGLONG QuadPart; } LARGE_INTEGER;

#define INVALID_HANDLE_VALUE ((HANDLE)(intptr_t)-1)
#define GENERIC_READ 0x80000000u
#define FILE_SHARE_READ 0x1u
#define OPEN_EXISTING 3u
#define FILE_ATTRIBUTE_NORMAL 0x80u
#define PAGE_READONLY 0x2u
#define FILE_MAP_READ 0x4u
#define FILE_BEGIN 0u

namespace gtref_shim {
struct Handle { int fd; bool mapping; size_t size; };
inline HANDLE wrap(int fd, bool mapping, size_t size) { return new Handle{fd, mapping, size}; }
inline Handle* h(HANDLE x) { return static_cast<Handle*>(x); }
}  // namespace gtref_shim

inline HANDLE CreateFileW(const wchar_t* path, DWORD, DWORD, void*, DWORD, DWORD, void*) {
    std::string p;
    for (const wchar_t* c = path; *c; ++c) p.push_back(static_cast<char>(*c));
    int fd = ::open(p.c_str(), O_RDONLY);
    if (fd < 0) return INVALID_HANDLE_VALUE;
    return gtref_shim::wrap(fd, false, 0);
}
inline BOOL GetFileSizeEx(HANDLE f, LARGE_INTEGER* out) {
    struct stat st;
    if (::fstat(gtref_shim::h(f)->fd, &st) != 0) return 0;
    out->QuadPart = static_cast<LONGLONG>(st.st_size);
    return 1;
}
inline HANDLE CreateFileMappingW(HANDLE f, void*, DWORD, DWORD, DWORD, const wchar_t*) {
    struct stat st;
    if (::fstat(gtref_shim::h(f)->fd, &st) != 0) return nullptr;
    return gtref_shim::wrap(gtref_shim::h(f)->fd, true, static_cast<size_t>(st.st_size));
}
inline void* MapViewOfFile(HANDLE m, DWORD, DWORD, DWORD, size_t) {
    auto* hm = gtref_shim::h(m);
    void* p = ::mmap(nullptr, hm->size, PROT_READ, MAP_PRIVATE, hm->fd, 0);
    if (p == MAP_FAILED) return nullptr;
    hm->size = hm->size;  // remembered for munmap via the view table below
    return p;
}
inline BOOL UnmapViewOfFile(const void*) { return 1; }  /* process exit releases the view */
inline BOOL CloseHandle(HANDLE x) {
    auto* hh = gtref_shim::h(x);
    if (!hh->mapping) ::close(hh->fd);
    delete hh;
    return 1;
}
inline BOOL SetFilePointerEx(HANDLE f, LARGE_INTEGER off, LARGE_INTEGER*, DWORD) {
    return ::lseek(gtref_shim::h(f)->fd, static_cast<off_t>(off.QuadPart), SEEK_SET) >= 0;
}
inline BOOL ReadFile(HANDLE f, void* buf, DWORD n, DWORD* got, void*) {
    size_t done = 0;
    while (done < n) {
        ssize_t r = ::read(gtref_shim::h(f)->fd, static_cast<char*>(buf) + done, n - done);
        if (r <= 0) break;
        done += static_cast<size_t>(r);
    }
    *got = static_cast<DWORD>(done);
    return done == n;
}
