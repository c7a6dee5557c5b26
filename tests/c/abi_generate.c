/*
 * The C ABI by itself: this program includes only include/graphgp_b200.h (plus the CUDA
 * runtime for device memory), links libgraphgp_b200.so, and runs
 *   gpb2_problem_create -> gpb2_generate -> gpb2_generate_logdet -> gpb2_problem_destroy
 * on a problem read from raw files, writing the field and the log-determinant to a file.
 * With no GPU arguments it only exercises the host entry points (version, the sharding plan,
 * the host graph build and an error path), which need no device.
 *
 * usage: abi_generate host
 *        abi_generate gpu <dir>    (dir holds meta.txt, coords.u32, nbrs.i64, offsets.i64,
 *                                   indices.i64, bins.f64, vals.f64, xi.f64; writes out.f64)
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "graphgp_b200.h"

#ifdef WITH_CUDA
#include <cuda_runtime.h>
#endif

static int fail(const char* what, int rc) {
    fprintf(stderr, "%s failed (%d): %s\n", what, rc, gpb2_last_error());
    return 1;
}

#ifdef WITH_CUDA
static void* read_all(const char* dir, const char* name, size_t* bytes) {
    char path[4096];
    snprintf(path, sizeof(path), "%s/%s", dir, name);
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void* buf = malloc((size_t)n > 0 ? (size_t)n : 1);
    if (fread(buf, 1, (size_t)n, f) != (size_t)n) {
        fclose(f);
        free(buf);
        return NULL;
    }
    fclose(f);
    *bytes = (size_t)n;
    return buf;
}
#endif

static int host_checks(void) {
    if (gpb2_version() != GPB2_VERSION) return fail("gpb2_version", gpb2_version());
    /* An invalid call returns a status and leaves a message; nothing aborts. */
    gpb2_graph* g = NULL;
    int rc = gpb2_build_graph(NULL, 10, 2, 1, 2, 4, 21, 1, &g);
    if (rc != GPB2_ERR_INVALID_ARG || strlen(gpb2_last_error()) == 0) return fail("error path", rc);
    /* The sharding plan of rank 1 of 2 over batches [4, 10), [10, 20000). */
    int64_t offs[3] = {4, 10, 20000}, flo[2], fhi[2], olo[2], ohi[2], slack = -1;
    int sh[2];
    rc = gpb2_shard_plan(offs, 3, 2, 1, 100, flo, fhi, olo, ohi, sh, &slack);
    if (rc != GPB2_OK) return fail("gpb2_shard_plan", rc);
    if (sh[0] != 0 || sh[1] != 1 || flo[1] != 10005 || fhi[1] != 20000 || olo[0] != 7 ||
        ohi[0] != 10 || slack != 0)
        return fail("gpb2_shard_plan values", -1);
    /* A small host graph build. */
    enum { N = 500, D = 2 };
    double* pts = (double*)malloc(sizeof(double) * N * D);
    uint64_t s = 12345;
    for (int i = 0; i < N * D; i++) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        pts[i] = (double)(s >> 11) / 9007199254740992.0;
    }
    rc = gpb2_build_graph(pts, N, D, 0, 20, 6, 21, 1, &g);
    free(pts);
    if (rc != GPB2_OK) return fail("gpb2_build_graph", rc);
    int64_t nof = gpb2_graph_n_offsets(g), n0 = gpb2_graph_n0(g);
    int64_t* of = (int64_t*)malloc(sizeof(int64_t) * nof);
    double scale = 0;
    rc = gpb2_graph_export(g, NULL, NULL, NULL, of, &scale);
    gpb2_graph_free(g);
    if (rc != GPB2_OK || of[0] != n0 || of[nof - 1] != N || !(scale > 0)) {
        free(of);
        return fail("gpb2_graph_export", rc);
    }
    free(of);
    printf("host ok\n");
    return 0;
}

#ifdef WITH_CUDA
static int gpu_checks(const char* dir) {
    size_t nb_meta = 0;
    char* meta = (char*)read_all(dir, "meta.txt", &nb_meta);
    if (!meta) return fail("meta.txt", -1);
    long long n, d, k, n0, noff, nbins;
    double scale;
    if (sscanf(meta, "%lld %lld %lld %lld %lld %lld %lf", &n, &d, &k, &n0, &noff, &nbins, &scale) != 7)
        return fail("meta.txt parse", -1);
    free(meta);
    size_t b1, b2, b3, b4, b5, b6, b7;
    uint32_t* coords = (uint32_t*)read_all(dir, "coords.u32", &b1);
    int64_t* nbrs = (int64_t*)read_all(dir, "nbrs.i64", &b2);
    int64_t* offsets = (int64_t*)read_all(dir, "offsets.i64", &b3);
    int64_t* indices = (int64_t*)read_all(dir, "indices.i64", &b4);
    double* bins = (double*)read_all(dir, "bins.f64", &b5);
    double* vals = (double*)read_all(dir, "vals.f64", &b6);
    double* xi = (double*)read_all(dir, "xi.f64", &b7);
    if (!coords || !nbrs || !offsets || !indices || !bins || !vals || !xi)
        return fail("inputs", -1);
    void *dc, *dn, *db, *dv, *dx, *dout;
    cudaMalloc(&dc, b1);
    cudaMalloc(&dn, b2);
    cudaMalloc(&db, b5);
    cudaMalloc(&dv, b6);
    cudaMalloc(&dx, b7);
    cudaMalloc(&dout, b7);
    cudaMemcpy(dc, coords, b1, cudaMemcpyHostToDevice);
    cudaMemcpy(dn, nbrs, b2, cudaMemcpyHostToDevice);
    cudaMemcpy(db, bins, b5, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, vals, b6, cudaMemcpyHostToDevice);
    cudaMemcpy(dx, xi, b7, cudaMemcpyHostToDevice);
    gpb2_problem* p = NULL;
    int rc = gpb2_problem_create(&p, GPB2_F64, 0, (const uint32_t*)dc, d, n, dn, 8, 0, k, offsets,
                                 noff, n0, scale, db, dv, nbins, indices, 0, NULL);
    if (rc != GPB2_OK) return fail("gpb2_problem_create", rc);
    rc = gpb2_generate(p, dx, dout, NULL);
    if (rc != GPB2_OK) return fail("gpb2_generate", rc);
    double ld = 0;
    rc = gpb2_generate_logdet(p, &ld, NULL);
    if (rc != GPB2_OK) return fail("gpb2_generate_logdet", rc);
    rc = gpb2_problem_destroy(p);
    if (rc != GPB2_OK) return fail("gpb2_problem_destroy", rc);
    double* out = (double*)malloc(b7 + sizeof(double));
    cudaMemcpy(out, dout, b7, cudaMemcpyDeviceToHost);
    out[n] = ld;
    char path[4096];
    snprintf(path, sizeof(path), "%s/out.f64", dir);
    FILE* f = fopen(path, "wb");
    fwrite(out, sizeof(double), (size_t)n + 1, f);
    fclose(f);
    printf("gpu ok\n");
    return 0;
}
#endif

int main(int argc, char** argv) {
    if (argc >= 2 && strcmp(argv[1], "host") == 0) return host_checks();
#ifdef WITH_CUDA
    if (argc >= 3 && strcmp(argv[1], "gpu") == 0) return host_checks() || gpu_checks(argv[2]);
#endif
    fprintf(stderr, "usage: %s host | gpu <dir>\n", argv[0]);
    return 2;
}
