/* A stand-in for the NCCL entry points that bh_tp_* resolve at run time,
 * for host-only tests of their bounded waits (built by tests/test_tp_comm.py
 * and loaded through BH_NCCL_LIB). A "unique id" names a rendezvous
 * directory; each rank that calls ncclCommInitRankConfig leaves a file there,
 * and a communicator stays in progress until every rank of the world has
 * done so. ncclCommAbort leaves an "aborted_<rank>" file, so a test can see
 * that a timed-out communicator was aborted. Collectives are not provided
 * (ncclInvalidUsage). Types are the C ABI's: results are int, communicators
 * are pointers, the unique id is 128 bytes passed by value. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct { char internal[128]; } fake_id;
typedef struct {
    char dir[128];
    int nranks, rank;
} fake_comm;

enum { OK = 0, INTERNAL = 3, INVALID_USAGE = 5, IN_PROGRESS = 7 };

static void touch(const char* dir, const char* name, int rank) {
    char path[256];
    snprintf(path, sizeof path, "%s/%s_%d", dir, name, rank);
    FILE* f = fopen(path, "w");
    if (f) fclose(f);
}

int ncclGetUniqueId(fake_id* id) {
    char tmpl[] = "/tmp/fake_nccl_XXXXXX";
    if (!mkdtemp(tmpl)) return INTERNAL;
    memset(id, 0, sizeof *id);
    strncpy(id->internal, tmpl, sizeof id->internal - 1);
    return OK;
}

int ncclCommInitRankConfig(fake_comm** comm, int nranks, fake_id id, int rank, void* config) {
    (void)config;
    fake_comm* c = (fake_comm*)calloc(1, sizeof *c);
    if (!c) return INTERNAL;
    memcpy(c->dir, id.internal, sizeof c->dir);
    c->dir[sizeof c->dir - 1] = 0;
    c->nranks = nranks;
    c->rank = rank;
    touch(c->dir, "rank", rank);
    *comm = c;
    return IN_PROGRESS;
}

int ncclCommGetAsyncError(fake_comm* c, int* state) {
    char path[256];
    struct stat sb;
    for (int r = 0; r < c->nranks; ++r) {
        snprintf(path, sizeof path, "%s/rank_%d", c->dir, r);
        if (stat(path, &sb) != 0) {
            *state = IN_PROGRESS;
            return OK;
        }
    }
    *state = OK;
    return OK;
}

int ncclCommAbort(fake_comm* c) {
    touch(c->dir, "aborted", c->rank);
    free(c);
    return OK;
}

int ncclCommFinalize(fake_comm* c) { (void)c; return OK; }
int ncclCommDestroy(fake_comm* c) { free(c); return OK; }
int ncclCommCount(const fake_comm* c, int* n) { *n = c->nranks; return OK; }
int ncclCommUserRank(const fake_comm* c, int* r) { *r = c->rank; return OK; }
int ncclAllGather(const void* s, void* r, size_t n, int t, fake_comm* c, void* st) {
    (void)s; (void)r; (void)n; (void)t; (void)c; (void)st;
    return INVALID_USAGE;
}
int ncclAllReduce(const void* s, void* r, size_t n, int t, int op, fake_comm* c, void* st) {
    (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st;
    return INVALID_USAGE;
}
