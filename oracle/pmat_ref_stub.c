/*
 * TEST INFRASTRUCTURE ONLY. The reference's packed matvec (src/vx27_pmat.c:229-244) first
 * offers BP3 rows to its Vulkan path through vx27_gpu_reg_matvec (src/vx27_gpu_reg.c,
 * which needs a Vulkan loader this machine does not have) and falls back to the CPU when
 * that returns anything but 1. This stub declines, so the reference's own CPU kernels run.
 */
int vx27_gpu_reg_matvec(const void *W, int rows, int cols, const float *x, float *y,
                        double *ms);
int vx27_gpu_reg_matvec(const void *W, int rows, int cols, const float *x, float *y,
                        double *ms) {
    (void)W; (void)rows; (void)cols; (void)x; (void)y; (void)ms;
    return 0;
}
