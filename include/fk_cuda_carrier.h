/* fk_cuda_carrier.h -- the handle door, as the CUDA carrier implements it.
 *
 * These are exactly the weak symbols the reference runtime declares (runtime/fkwu-uni.c:910-1009)
 * and its Metal carrier defines (form/native/metal/fk-metal-carrier.m).  Linking the carrier object
 * into the runtime overrides the weak stubs; Form's metal_* primitives (runtime/fkwu-optable.h:91-104)
 * then reach sm_100a kernels.  Handles are (generation << 16) | slot with slot 1-based; 0 is never a
 * live handle.  Each call answers as its Metal counterpart does (cited per line) and records a
 * last_error string that fk_metal_status_external reports.
 */
#ifndef FK_CUDA_CARRIER_H
#define FK_CUDA_CARRIER_H

#ifdef __cplusplus
extern "C" {
#endif

/* fk-metal-carrier.m:447  -- resolve `name` to a registered sm_100a kernel; same text + name = same handle; 0 on refusal */
long long fk_metal_pipeline_external(const char *msl, long long msl_len, const char *name, long long name_len);
/* fk-metal-carrier.m:561  -- zero-filled device buffer of nbytes; 0 on refusal */
long long fk_metal_buf_alloc_external(long long nbytes);
/* fk-metal-carrier.m:580  -- the file region [off, off+len) copied into device memory once; len < 0 = a
 * writable region of a shared file, written back at every sync */
long long fk_metal_buf_from_file_external(const char *path, long long path_len, long long off, long long len);
/* fk-metal-carrier.m:658  -- stream-ordered write of len bytes at off; answers len or -1 */
long long fk_metal_buf_write_external(long long h, long long off, const char *bytes, long long len);
/* fk-metal-carrier.m:688  -- bind and dispatch without waiting; 1 or -1 */
long long fk_metal_enqueue_external(long long pipe, const char *binding, long long binding_len, long long threads);
/* fk-metal-carrier.m:851  -- drain everything; the number of dispatches drained, or -1 */
long long fk_metal_sync_external(void);
/* fk-metal-carrier.m:907  -- sync first, then exactly len bytes, or -1 (never a short read) */
long long fk_metal_buf_read_external(long long h, long long off, long long len, char *out, long long cap);
/* fk-metal-carrier.m:1039 -- key=value text: metal_linked=true, metal_door=handle, counters, last_error */
long long fk_metal_status_external(char *out, long long cap);
/* fk-metal-carrier.m:928  -- arm the next batch as concurrent (barrier_before then legal) */
long long fk_metal_batch_concurrent_external(void);
/* fk-metal-carrier.m:945  -- free at a quiescent point only; bumps the slot's generation */
long long fk_metal_buf_free_external(long long h);
/* fk-metal-carrier.m:977  -- close the open batch without waiting; a fence id, 0 if nothing to submit */
long long fk_metal_submit_external(void);
/* fk-metal-carrier.m:1013 -- wait for one fence; its dispatch count, 0 for an unknown fence, -1 on error */
long long fk_metal_fence_wait_external(long long fence);
/* fk-metal-carrier.m:192, :208 -- the one-shot text doors (fkwu-uni.c:910-929) */
long long fk_metal_matvec_fixture_external(char *out, long long cap);
long long fk_metal_matvec_f32_external(const char *msl, long long msl_len, const char *kernel, long long kernel_len,
                                       const char *model, long long model_len, char *out, long long cap);

/* ---- the CUDA matvec doors, tag 232 (fixture witness) and tag 233 `(cuda_matvec_f32 W x)`, which the
 * reference serves only on Windows through nvcuda.dll (runtime/fkwu-uni.c:4753-5050).
 * fkwu-uni.c:4764 fk_cuda_go -- y = W.x with W [rows*cols], x [cols], y [rows] in HOST memory, one
 * device thread per row folding j downward with two roundings per term (no fused multiply-add);
 * the device name into gname.  0, or the first refusal's negative code (-3 no driver, -4 no device,
 * -9 launch failed, -10 device allocation or copy failed). */
long long fk_cuda_go_external(const float *W, const float *x, float *y, unsigned rows, unsigned cols, char *gname,
                              long long gcap);
/* fkwu-uni.c:4976 fk_cuda_matvec_f32 -- the tag-233 door's work: fk_cuda_go, then the same fold on the
 * CPU; answers the number of rows that agree bit for bit (the `agree` head of the returned list), or
 * a negative code; -1 for the door's own refusals (cols == 0, more than 4194304 weights). */
long long fk_cuda_matvec_f32_external(const float *W, const float *x, float *y, unsigned rows, unsigned cols);
/* fkwu-uni.c:4907 fk_cuda_matvec -- tag 232: the fixed 3x4 witness; answers the rows that agree (3) */
long long fk_cuda_matvec_fixture_external(void);

#ifdef __cplusplus
}
#endif
#endif
