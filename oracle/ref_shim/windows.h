/*
 * Minimal stand-in for <windows.h> so that the reference's CPU arithmetic in
 * src/p8c_segmented_access_correctness.cpp can be compiled in place on Linux
 * by oracle/build.py.  Only the names that file mentions are declared; the
 * Vulkan/Win32 code paths that use them are never called by the oracle
 * wrapper (oracle/ref_wrap.cpp).  TEST INFRASTRUCTURE ONLY.
 */
#pragma once
#define WINAPI
typedef void *HMODULE;
typedef void *FARPROC;
static inline HMODULE LoadLibraryA(const char *) { return nullptr; }
static inline FARPROC GetProcAddress(HMODULE, const char *) { return nullptr; }
static inline int FreeLibrary(HMODULE) { return 0; }
