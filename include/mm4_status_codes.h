/* Status codes shared by the mm4 C ABI and its device code. The reference
 * reports failures as NSError codes at session init and fatalError at
 * dispatch (ConvolutionShared.swift:869-907, :955-958); mm4 returns them. */
#ifndef MM4_STATUS_CODES_H
#define MM4_STATUS_CODES_H

#define MM4_OK 0
#define MM4_ERR_INVALID 1     /* bad descriptor, null pointer, unsupported value */
#define MM4_ERR_UNSUPPORTED 2 /* valid request this build does not implement */
#define MM4_ERR_CUDA 3        /* CUDA runtime/driver error or no sm_100 device */
#define MM4_ERR_NCCL 4        /* collective failure (multi-GPU paths) */
#define MM4_ERR_TIMEOUT 5     /* a device-side bounded wait ran out */
#define MM4_ERR_WORKSPACE 6   /* workspace missing or too small */

#endif
