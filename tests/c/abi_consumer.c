/* A plain-C caller of libhar_cuda.so, built by tests/test_c_consumer.py with
 * gcc against include/har_cuda.h only: the ABI a Rust FFI crate binds is usable
 * from C with no other header.  Without a GPU it checks the fail-closed
 * context creation; with a GGUF path it reads the file's directory (host-only).
 * Prints one line of key=value pairs; exit status 0 when every check held. */
#include <stdio.h>
#include <string.h>

#include "har_cuda.h"

int main(int argc, char **argv) {
  int ok = 1;
  const int32_t ver = har_cuda_abi_version();
  har_cuda_ctx *ctx = NULL;
  const int32_t st = har_cuda_ctx_create(0, &ctx);
  printf("abi=%d ctx_status=%d", ver, st);
  if (ver != HAR_CUDA_ABI_VERSION) ok = 0;
  if (st == HAR_CUDA_OK) {
    har_cuda_ctx_destroy(ctx);
  } else if (ctx != NULL) {
    ok = 0; /* a failed create leaves no handle */
  }
  if (har_cuda_synchronize(NULL, 10) != HAR_CUDA_ERR_ARG) ok = 0;
  if (argc > 1) {
    char err[256];
    har_cuda_gguf *g = NULL;
    if (har_cuda_gguf_open(argv[1], err, sizeof err, &g) != HAR_CUDA_OK) {
      printf(" gguf_error=\"%s\"", err);
      ok = 0;
    } else {
      uint32_t version = 0;
      uint64_t tensors = 0, align = 0, data = 0;
      har_cuda_gguf_header(g, &version, &tensors, NULL, &align, &data);
      char name[128];
      uint32_t type = 0, rank = 0;
      uint64_t dims[16], off = 0, bytes = 0;
      har_cuda_gguf_tensor_info(g, 0, name, sizeof name, &type, &rank, dims, &off, &bytes);
      printf(" version=%u tensors=%llu alignment=%llu name=%s type=%u rank=%u payload=%llu",
             version, (unsigned long long)tensors, (unsigned long long)align, name, type, rank,
             (unsigned long long)bytes);
      if (har_cuda_gguf_find(g, name) != 0) ok = 0;
      har_cuda_gguf_close(g);
    }
  }
  printf(" ok=%d\n", ok);
  return ok ? 0 : 1;
}
