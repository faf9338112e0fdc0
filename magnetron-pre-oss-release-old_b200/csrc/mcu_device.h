/* Device state that host modules other than device.c use (storage.c). */
#ifndef MCU_DEVICE_H
#define MCU_DEVICE_H

#include "mag_cuda_abi.h"

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

int mcu_dev_ordinal(mag_compute_device_t* dvc);
/* Waits for the device stream; returns a CUDA error or a kernel status code. */
int mcu_dev_sync(mag_compute_device_t* dvc);
/* Buffer bookkeeping for data read (p) or written (bytes at p) outside the device stream's ops. */
void mcu_dev_in(mag_compute_device_t* dvc, const void* p);
void mcu_dev_out(mag_compute_device_t* dvc, void* p, size_t bytes);

#ifdef __cplusplus
}
#endif
#endif
