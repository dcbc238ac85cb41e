/* Status codes returned by every vireo-b200 C-ABI call that can fail.
 * (The reference's gguf_compute.h / expert_store.h calls return nothing or
 * -1; the drop-in versions keep their signatures and report details through
 * vireo_last_error().) */
#ifndef VIREO_STATUS_H
#define VIREO_STATUS_H

#define VIREO_OK 0
#define VIREO_ERR_ARG (-1)         /* bad argument / shape / alignment      */
#define VIREO_ERR_CUDA (-2)        /* a CUDA runtime call failed             */
#define VIREO_ERR_UNSUPPORTED (-3) /* tensor type or shape not implemented   */
#define VIREO_ERR_TIMEOUT (-4)     /* a bounded device wait ran out          */
#define VIREO_ERR_NOMEM (-5)       /* device or pinned-host allocation failed */
#define VIREO_ERR_IO (-6)          /* pread from the backing file failed      */
#define VIREO_ERR_NODEV (-7)       /* no usable CUDA device                   */

#endif
