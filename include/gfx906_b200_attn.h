/*
 * C ABI of the B200 (sm_100a) flash-attention forward path.
 *
 * Drop-in for the reference's kernel shim: the reference binds
 *   extern "C" void launch(const void*, const void*, const void*, void*,
 *                          int, int, int, int, int, float, hipStream_t);
 * (attn_kernel.hip:710-711, declared again in attn.cpp:4-5). This library
 * exports the same symbol with the same argument order and meaning, with a
 * CUDA stream in place of the HIP stream, plus a status-returning form.
 *
 * Tensors: q [B,H,Sq,D], k and v [B,H,Skv,D], o [B,H,Sq,D]; fp16 (IEEE
 * binary16), contiguous, device pointers, 16-byte aligned. The caller owns
 * every buffer (the library allocates nothing per call). Work is enqueued
 * asynchronously on `stream`; nothing synchronises.
 * Supported head dims: D <= 64 with D % 8 == 0, D == 128, D == 512
 * (the reference's envelope, attn.cpp:13-14).
 * Skv == 0 writes zeros to o (the reference left such rows unwritten).
 * Only sm_100 devices (B200) are accepted.
 */
#ifndef GFX906_B200_ATTN_H
#define GFX906_B200_ATTN_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define GFX906_B200_API __attribute__((visibility("default")))
#else
#define GFX906_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by gfx906_b200_attn_launch. */
#define GFX906_B200_OK 0
#define GFX906_B200_EINVAL 1      /* negative size, null pointer, size overflow */
#define GFX906_B200_EHEADDIM 2    /* D not in {8,16,...,64, 128, 512} */
#define GFX906_B200_EALIGN 3      /* a pointer is not 16-byte aligned */
#define GFX906_B200_ENODEV 4      /* current device is not sm_100 */
#define GFX906_B200_ECUDA 5       /* a CUDA runtime or driver call failed */
#define GFX906_B200_ETIMEOUT 6    /* a kernel wait ran out (device status word) */
#define GFX906_B200_ENOSPACE 7    /* needs more scratch than the built-in array holds */

/* Replaces attn_kernel.hip:710-742 `launch` (same arguments; cudaStream_t for
 * hipStream_t). Returns nothing, like the reference; the status of the call
 * is kept for gfx906_b200_attn_last_error(). */
GFX906_B200_API void launch(const void* q, const void* k, const void* v, void* o,
            int B, int H, int Sq, int Skv, int D, float scale,
            cudaStream_t stream);

/* Same work as launch(); returns a GFX906_B200_* status instead of void.
 * The reference's launch never checks its arguments or launch errors
 * (attn_kernel.hip:710-742); this form reports both. */
GFX906_B200_API int gfx906_b200_attn_launch(const void* q, const void* k, const void* v,
                            void* o, int B, int H, int Sq, int Skv, int D,
                            float scale, cudaStream_t stream);

/* Bytes of workspace gfx906_b200_attn_launch_ws needs for these sizes on the
 * current device (0 when the call does not split work across CTAs). No
 * reference counterpart: the reference's kernels keep nothing between CTAs. */
GFX906_B200_API size_t gfx906_b200_attn_workspace_size(int B, int H, int Sq, int Skv, int D);

/* Same work as gfx906_b200_attn_launch, with a caller-owned device workspace
 * that lets the kernel balance the key range of every (batch, head, query
 * block) across all SMs (partial results are combined on the GPU). The
 * workspace must be 256-byte aligned and at least
 * gfx906_b200_attn_workspace_size() bytes; its contents on entry do not
 * matter (a call reads only the partial results it wrote itself, and its
 * arrival counters carry a per-launch tag), so it needs
 * no clearing and may be reused for calls of any size. Calls that share a
 * workspace must not overlap on the GPU (use one stream, or one workspace per
 * stream). Extension of attn_kernel.hip:710-742 (same arguments plus the
 * workspace). */
GFX906_B200_API int gfx906_b200_attn_launch_ws(const void* q, const void* k, const void* v,
                               void* o, int B, int H, int Sq, int Skv, int D,
                               float scale, void* workspace, size_t workspace_bytes,
                               cudaStream_t stream);

/* Schedule that gfx906_b200_attn_launch (with_workspace == 0) or
 * gfx906_b200_attn_launch_ws (with_workspace != 0) picks for these sizes on
 * a GPU with num_sms SMs (num_sms <= 0: the current device, which must then
 * be an sm_100 GPU; num_sms > 0 touches no GPU): out4[0] = CTAs launched,
 * out4[1] = 0 for whole units, 1 when the key range is split across CTAs and
 * the pieces are combined inside the attention kernel, 2 when they are
 * combined by a second kernel launched after it, out4[2] = CTAs sharing the
 * split key range, out4[3] = query rows per work unit (128 or 256). All zero when nothing is launched (an empty problem, Skv == 0).
 * Returns a GFX906_B200_* status. No reference counterpart: the reference's
 * grid is always (B*H, ceil(Sq/64)) (attn_kernel.hip:714-741). */
GFX906_B200_API int gfx906_b200_attn_plan(int B, int H, int Sq, int Skv, int D,
                          int with_workspace, int num_sms, int* out4);

/* Caps the SMs the persistent kernels plan for, process-wide: launches after
 * this call use at most `sms` CTAs (D = 512: sms / 2 two-CTA clusters, at
 * least one), and gfx906_b200_attn_workspace_size and
 * gfx906_b200_attn_plan(num_sms = 0) follow the cap. sms <= 0 removes it.
 * Returns the previous cap (0 = none). The SMs left over run kernels of
 * other streams beside the attention kernel -- the NCCL broadcast of the
 * next call's K/V and the gather of the previous call's output in a sharded
 * pipeline -- which otherwise wait until the all-SM kernel ends. Set it
 * while no other thread is between workspace_size and launch_ws. No
 * reference counterpart (the reference has no persistent grid). */
GFX906_B200_API int gfx906_b200_attn_set_sm_limit(int sms);

/* Allocation-free form of gfx906_b200_attn_launch_ws, for callers that cannot
 * allocate device memory (a plugin whose host runtime owns all device memory,
 * an application with a fixed memory budget, a latency-critical path where
 * cudaMalloc/cudaFree would lock or synchronise). Its scratch is a fixed
 * array of gfx906_b200_attn_noalloc_capacity() bytes (48 MiB) compiled into
 * the library; a GPU holds it from the first call on that device until the
 * process exits. That first call looks up the array's device address and
 * should come before any stream capture on the device. Calls whose split
 * schedule needs more scratch return GFX906_B200_ENOSPACE; the scratch a
 * schedule needs grows with the device's SM count (at most ~40 MB on a
 * 148-SM B200, so no call on a B200 gets ENOSPACE). All calls on a device
 * share the array: calls that overlap on the GPU race, so order them on one
 * stream. Allocates nothing. No counterpart in the reference. */
GFX906_B200_API int gfx906_b200_attn_launch_noalloc(const void* q, const void* k, const void* v,
                                    void* o, int B, int H, int Sq, int Skv, int D,
                                    float scale, cudaStream_t stream);

/* Same attention with every (batch, head) matrix stored transposed: q and o
 * are [B, H, D, Sq], k and v [B, H, D, Skv], contiguous, the sequence
 * innermost. A [b, c, h, w] feature map is this layout with H = 1, D = c and
 * S = h * w, so the VAE mid-block attention (deploy/gfx906_attention.py:82-111
 * in the reference, which transposes to [b, 1, h*w, c] and back around
 * launch) runs on the feature maps as they are. D must be 512
 * (GFX906_B200_EHEADDIM otherwise); Sq and Skv must be multiples of 8 so that
 * every row starts on 16 bytes (GFX906_B200_EALIGN otherwise). */
GFX906_B200_API int gfx906_b200_attn_launch_dmajor(const void* q, const void* k, const void* v,
                                   void* o, int B, int H, int Sq, int Skv, int D,
                                   float scale, cudaStream_t stream);

/* Size in bytes of the scratch array behind gfx906_b200_attn_launch_noalloc.
 * No counterpart in the reference. */
GFX906_B200_API size_t gfx906_b200_attn_noalloc_capacity(void);

/* Status of the last launch()/gfx906_b200_attn_launch() on this host thread.
 * No reference counterpart (the reference's launch returns void). */
GFX906_B200_API int gfx906_b200_attn_last_error(void);

/* Human-readable text for a GFX906_B200_* status. No reference counterpart. */
GFX906_B200_API const char* gfx906_b200_attn_error_string(int status);

/* Reads (and, if reset != 0, clears) the device status word of the current
 * device, which a kernel sets when one of its bounded waits runs out.
 * Synchronises the device. Returns GFX906_B200_OK or GFX906_B200_ETIMEOUT
 * (GFX906_B200_ECUDA if the read itself fails). No reference counterpart:
 * the reference's kernels have no waits that can time out. */
GFX906_B200_API int gfx906_b200_attn_device_status(int reset);

/* Diagnostics of the first timed-out wait since the last reset:
 * out[0]=block x, out[1]=block y, out[2]=warp, out[3]=barrier index,
 * out[4]=phase parity, out[5]=role. Synchronises. Returns a status. */
GFX906_B200_API int gfx906_b200_attn_timeout_info(int* out6);

/* Self-test of the bounded wait: launches one block that waits on an
 * mbarrier nothing arrives at, with the given limit in nanoseconds. The
 * block gives up, sets the device status word and exits, leaving the
 * context usable. Used by the GPU tests of failure detection. No reference
 * counterpart. */
GFX906_B200_API int gfx906_b200_attn_selftest_wait_timeout(unsigned long long timeout_ns,
                                           cudaStream_t stream);

/* Floating-point operations of one call, 4*B*H*Sq*Skv*D, the reference's
 * throughput formula (flops_probe.py:18). */
GFX906_B200_API double gfx906_b200_attn_flops(int B, int H, int Sq, int Skv, int D);

#ifdef __cplusplus
}
#endif

#endif /* GFX906_B200_ATTN_H */
