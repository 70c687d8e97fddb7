//! The C ABI of libforgesort.so (include/forgesort.h, include/forgesort_bench.h).
//!
//! Replaces forge-sort's Metal layer (src/metal_helpers.rs: device, queue,
//! buffers, pipeline states).  Every function returns an `fs_status`
//! (0 = success); `fs_last_error` gives the text of the last failure.
//!
//! NOT COMPILED: no cargo / rustc on the image this was written on.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

#[repr(C)]
pub struct FsSorter {
    _p: [u8; 0],
}
#[repr(C)]
pub struct FsBuffer {
    _p: [u8; 0],
}
#[repr(C)]
pub struct FsMg {
    _p: [u8; 0],
}

// fs_dtype
pub const FS_U32: c_int = 0;
pub const FS_I32: c_int = 1;
pub const FS_F32: c_int = 2;
pub const FS_U64: c_int = 3;
pub const FS_I64: c_int = 4;
pub const FS_F64: c_int = 5;

// fs_status
pub const FS_OK: c_int = 0;
pub const FS_E_DEVICE_NOT_FOUND: c_int = 1;
pub const FS_E_KERNEL_IMAGE: c_int = 2;
pub const FS_E_GPU_EXECUTION: c_int = 3;
pub const FS_E_LENGTH_MISMATCH: c_int = 4;
pub const FS_E_TIMEOUT: c_int = 5;
pub const FS_E_NCCL: c_int = 6;
pub const FS_E_OOM: c_int = 7;
pub const FS_E_INVALID: c_int = 8;

extern "C" {
    // lifetime (GpuSorter::new / with_context, src/lib.rs:596-686)
    pub fn fs_create(device: c_int, stream: *mut c_void, out: *mut *mut FsSorter) -> c_int;
    pub fn fs_destroy(s: *mut FsSorter) -> c_int;
    pub fn fs_last_error(s: *const FsSorter) -> *const c_char;
    pub fn fs_set_stream(s: *mut FsSorter, stream: *mut c_void) -> c_int;
    pub fn fs_synchronize(s: *mut FsSorter) -> c_int;

    // SortBuffer objects (src/lib.rs:160-281, 694-785)
    pub fn fs_buffer_create(s: *mut FsSorter, bytes: u64, out: *mut *mut FsBuffer) -> c_int;
    pub fn fs_buffer_destroy(b: *mut FsBuffer) -> c_int;
    pub fn fs_buffer_host(b: *const FsBuffer) -> *mut c_void;
    pub fn fs_buffer_device(b: *const FsBuffer) -> *mut c_void;
    pub fn fs_buffer_bytes(b: *const FsBuffer) -> u64;
    pub fn fs_buffer_host_read(b: *mut FsBuffer) -> c_int;
    pub fn fs_buffer_host_write(b: *mut FsBuffer) -> c_int;
    pub fn fs_buffer_device_use(b: *mut FsBuffer, bytes: u64) -> c_int;
    pub fn fs_sort_buffer(s: *mut FsSorter, dtype: c_int, keys: *mut FsBuffer, n: u64, sync: c_int) -> c_int;
    pub fn fs_sort_pairs_buffer(s: *mut FsSorter, dtype: c_int, keys: *mut FsBuffer, vals: *mut FsBuffer, n: u64,
                                sync: c_int) -> c_int;

    // host slices (src/lib.rs:791-3015)
    pub fn fs_host_sort_keys(s: *mut FsSorter, dtype: c_int, keys: *mut c_void, n: u64) -> c_int;
    pub fn fs_host_sort_pairs(s: *mut FsSorter, dtype: c_int, keys: *mut c_void, nk: u64, vals: *mut u32,
                              nv: u64) -> c_int;
    pub fn fs_host_argsort(s: *mut FsSorter, dtype: c_int, keys: *const c_void, idx: *mut u32, n: u64) -> c_int;
    pub fn fs_host_sort_keys_copy(s: *mut FsSorter, dtype: c_int, hin: *const c_void, hout: *mut c_void,
                                  n: u64) -> c_int;
    pub fn fs_host_sort_keys_copy_async(s: *mut FsSorter, dtype: c_int, hin: *const c_void, hout: *mut c_void,
                                        n: u64) -> c_int;

    // device pointers
    pub fn fs_alloc(s: *mut FsSorter, bytes: usize, managed: c_int, ptr: *mut *mut c_void) -> c_int;
    pub fn fs_free(s: *mut FsSorter, ptr: *mut c_void) -> c_int;
    pub fn fs_sort_keys(s: *mut FsSorter, dtype: c_int, keys: *mut c_void, n: u64, sync: c_int) -> c_int;
    pub fn fs_sort_pairs(s: *mut FsSorter, dtype: c_int, keys: *mut c_void, vals: *mut u32, n: u64,
                         sync: c_int) -> c_int;
    pub fn fs_argsort(s: *mut FsSorter, dtype: c_int, keys: *const c_void, idx: *mut u32, n: u64,
                      sync: c_int) -> c_int;
    pub fn fs_sort_keys_copy(s: *mut FsSorter, dtype: c_int, kin: *const c_void, kout: *mut c_void, n: u64,
                             sync: c_int) -> c_int;
    pub fn fs_sort_pairs_copy(s: *mut FsSorter, dtype: c_int, kin: *const c_void, vin: *const u32,
                              kout: *mut c_void, vout: *mut u32, n: u64, sync: c_int) -> c_int;

    // forge-runtime: permutation apply and a context stream
    pub fn fs_gather(s: *mut FsSorter, width: c_int, src: *const c_void, src_n: u64, idx: *const u32,
                     dst: *mut c_void, n: u64, sync: c_int) -> c_int;
    pub fn fs_stream_create(device: c_int, stream: *mut *mut c_void) -> c_int;
    pub fn fs_stream_synchronize(stream: *mut c_void) -> c_int;
    pub fn fs_stream_destroy(stream: *mut c_void) -> c_int;

    // several GPUs of one process (no reference counterpart)
    pub fn fs_mg_create(devices: *const c_int, g: c_int, out: *mut *mut FsMg) -> c_int;
    pub fn fs_mg_destroy(mg: *mut FsMg) -> c_int;
    pub fn fs_mg_last_error(mg: *const FsMg) -> *const c_char;
    pub fn fs_mg_sort_keys(mg: *mut FsMg, dtype: c_int, shards: *const *mut c_void, shard_n: *const u64,
                           out: *const *mut c_void, out_cap: *const u64, out_n: *mut u64) -> c_int;
    pub fn fs_mg_sort_pairs(mg: *mut FsMg, dtype: c_int, shards: *const *mut c_void, vals: *const *const u32,
                            shard_n: *const u64, out: *const *mut c_void, out_vals: *const *mut u32,
                            out_cap: *const u64, out_n: *mut u64) -> c_int;

    // one process per GPU: sample-sort building blocks
    pub fn fs_partition_count_async(s: *mut FsSorter, dtype: c_int, keys: *const c_void, n: u64, gpos_base: u64,
                                    spl_keys: *const c_void, spl_gpos: *const u64, nsplit: c_int,
                                    counts_dev: *mut u64) -> c_int;
    pub fn fs_partition_dispatch_matrix(s: *mut FsSorter, dtype: c_int, keys: *const c_void, vals: *const u32,
                                        payload: c_int, n: u64, gpos_base: u64, spl_keys: *const c_void,
                                        spl_gpos: *const u64, nsplit: c_int, send_matrix: *const u64, rank: c_int,
                                        inbox_keys: *const *mut c_void, inbox_vals: *const *mut u32,
                                        sync: c_int) -> c_int;
    pub fn fs_ipc_export(s: *mut FsSorter, dev_ptr: *mut c_void, handle_out: *mut u8) -> c_int;
    pub fn fs_ipc_open(s: *mut FsSorter, handle: *const u8, peer_ptr: *mut *mut c_void) -> c_int;
    pub fn fs_ipc_close(s: *mut FsSorter, peer_ptr: *mut c_void) -> c_int;

    // a sort that allocates nothing (fixed in-library scratch, 4 MiB of keys)
    pub fn fs_sort_keys_noalloc(dtype: c_int, keys: *mut c_void, n: u64, stream: *mut c_void) -> c_int;

    pub fn fs_abi_version() -> c_int;
}
