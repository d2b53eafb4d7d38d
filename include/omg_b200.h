/*
 * omg_b200: C ABI of the B200 engine for the omg decision forward pass.
 *
 * This is the boundary a host-language shim binds (the reference's Rust
 * `omg_wgpu` crate would wrap it as an `extern "C"` block; see
 * INTEGRATION.md). Every entry point takes plain pointers and sizes, returns
 * 0 on success and -1 on error, and leaves a message for omg_last_error()
 * (thread-local, valid until the next call on the same thread). Outputs are
 * caller-allocated; nothing is written to them on error.
 *
 * Each declaration names the reference interface it replaces, as
 * `path:line` within github.com/bokuweb/omg.
 */
#ifndef OMG_B200_H
#define OMG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight storage types, numbered as model::Dtype::code
 * (crates/omg-wgpu/src/model.rs:357-363). */
enum { OMG_DTYPE_F16 = 0, OMG_DTYPE_Q8 = 1, OMG_DTYPE_Q4 = 2 };

/* omg_core::Want (crates/omg-core/src/backend.rs:15-20). */
enum { OMG_WANT_LOGITS = 0, OMG_WANT_HIDDEN = 1 };

/* omg_core::PrefixSource (crates/omg-core/src/backend.rs:95-104); NONE when
 * no pass has run yet. */
enum {
  OMG_SOURCE_NONE = -1,
  OMG_SOURCE_RESIDENT = 0,
  OMG_SOURCE_RAM = 1,
  OMG_SOURCE_DISK = 2,
  OMG_SOURCE_DECODED = 3
};

/* GEMM epilogues exposed to the kernel tests (gemm.cuh GemmEpilogue). */
enum { OMG_EPI_F32 = 0, OMG_EPI_GEGLU_TANH = 1, OMG_EPI_GEGLU_ERF = 2, OMG_EPI_F16 = 3 };

/* The message of the last failed call on this thread ("" if none). */
const char* omg_last_error(void);

/* Library version string. */
const char* omg_version(void);

/* ---- kernel-level entry points (parity tests) ------------------------------
 * Host buffers in and out; each call allocates its own device memory.
 */

/* Y = X * W^T on the tcgen05 GEMM: X [m, k] f16 (row stride lda), W [w_rows, k]
 * f16. epi OMG_EPI_F32 writes f32 [m, ldo] (split-K slabs summed on the host),
 * OMG_EPI_F16 writes f16 [m, ldo], the GeGLU epilogues expect W rows
 * interleaved in 256-row blocks [128 gate | 128 up] and write f16
 * act = gelu(g) * u for n_out columns. bn = 0 picks the engine's tiling.
 * Replaces crates/omg-wgpu/src/shaders/matmul.wgsl:1-9 and
 * matmul_gated.wgsl:1-7 (the tests of crates/omg-wgpu/tests/matmul.rs:201-290). */
int omg_debug_gemm(int device, const uint16_t* x_f16, int m, int k, int lda, const uint16_t* w_f16,
                   int w_rows, int n_out, int epi, int bn, int splits, void* out, int ldo);

#ifdef __cplusplus
}
#endif

#endif /* OMG_B200_H */
