/* TEST INFRASTRUCTURE: SBB1 blob reader and MT19937 for the C restatement.
 *
 * SBB1 layout (reference complete_port/pysim/sbb.py:1-53): 52-byte header
 * "SBB1", u32 version, u32 n_sections, u64 dir_off, u64 names_off, u64
 * names_len, u64 total, u64 reserved; 56-byte directory entries u32 name_off,
 * u32 dtype, u32 ndim, u32 reserved, u64 shape[4], u64 data_off. */
#include "sbo_internal.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static uint64_t ld64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }
static uint32_t ld32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }

int sbo_blob_open(SboBlob* b, const char* path) {
    memset(b, 0, sizeof(*b));
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 52) { close(fd); return -1; }
    void* m = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return -1;
    b->map = (uint8_t*)m;
    b->size = (size_t)st.st_size;
    if (memcmp(b->map, "SBB1", 4) != 0 || ld32(b->map + 4) != 1u) { sbo_blob_close(b); return -1; }
    b->nsec = (int)ld32(b->map + 8);
    const uint64_t dir = ld64(b->map + 12), names = ld64(b->map + 20);
    b->sec = (SboSec*)calloc((size_t)(b->nsec ? b->nsec : 1), sizeof(SboSec));
    for (int i = 0; i < b->nsec; i++) {
        const uint8_t* d = b->map + dir + (size_t)i * 56;
        SboSec* s = &b->sec[i];
        s->name = (const char*)(b->map + names + ld32(d));
        s->dtype = ld32(d + 4);
        s->ndim = ld32(d + 8);
        s->count = 1;
        for (uint32_t k = 0; k < s->ndim && k < 4; k++) s->count *= ld64(d + 16 + 8 * k);
        s->off = ld64(d + 48);
    }
    return 0;
}

void sbo_blob_close(SboBlob* b) {
    free(b->sec);
    if (b->map) munmap(b->map, b->size);
    memset(b, 0, sizeof(*b));
}

const SboSec* sbo_blob_find(const SboBlob* b, const char* name) {
    for (int i = 0; i < b->nsec; i++)
        if (strcmp(b->sec[i].name, name) == 0) return &b->sec[i];
    return NULL;
}

const void* sbo_blob_get(const SboBlob* b, const char* name, uint32_t dtype) {
    const SboSec* s = sbo_blob_find(b, name);
    return (s && s->dtype == dtype) ? (const void*)(b->map + s->off) : NULL;
}

double sbo_blob_f64_1(const SboBlob* b, const char* name, double dflt) {
    const double* p = (const double*)sbo_blob_get(b, name, 0);
    return p ? p[0] : dflt;
}

int64_t sbo_blob_i64_1(const SboBlob* b, const char* name, int64_t dflt) {
    const int64_t* p = (const int64_t*)sbo_blob_get(b, name, 2);
    return p ? p[0] : dflt;
}
