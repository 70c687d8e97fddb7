//! forge-sort on NVIDIA B200: the public API of metal-forge-compute/forge-sort
//! (src/lib.rs) over the CUDA library `libforgesort.so` (include/forgesort.h).
//!
//! NOT COMPILED: the image this was written on has no cargo / rustc, so this
//! crate has never been built.  Its behaviour is that of the C ABI, which the
//! repository's Python and C++ mirrors test on the GPU method for method.
//!
//! Differences from the Metal crate, all forced by the hardware:
//! - `with_context` takes a CUDA device ordinal and a `cudaStream_t` (as a raw
//!   pointer) instead of a Metal device and command queue; `encode_sort` takes
//!   a stream instead of a compute encoder.
//! - `SortBuffer<T>` is device memory plus a page-locked host mirror kept
//!   coherent by the library: sorts stay on the device, `as_slice` copies back
//!   only what sorts changed, `as_mut_slice` marks the device copy stale.  The
//!   borrow rules below (`&mut self` for writes) are what make this exact.
//! - `metal_buffer()` becomes `device_ptr()` (a deprecated alias is kept);
//!   `from_raw_parts` / `into_raw_parts` carry the library's buffer object.
//! - `SortError::DeviceNotFound` now means "no CUDA device"; its Display
//!   string is kept verbatim for source compatibility.

mod ffi;

use std::ffi::CStr;
use std::fmt;
use std::marker::PhantomData;
use std::os::raw::{c_int, c_void};
use std::ptr::NonNull;

mod private {
    pub trait Sealed {}
    impl Sealed for u32 {}
    impl Sealed for i32 {}
    impl Sealed for f32 {}
    impl Sealed for u64 {}
    impl Sealed for i64 {}
    impl Sealed for f64 {}
}

/// Types the GPU can radix-sort (sealed: u32, i32, f32, u64, i64, f64), with
/// the constants of forge-sort's trait (src/lib.rs:29-88).
pub trait SortKey: private::Sealed + Copy + 'static {
    const KEY_SIZE: usize;
    const NEEDS_TRANSFORM: bool;
    const IS_64BIT: bool;
    const TRANSFORM_MODE_FORWARD: u32;
    const TRANSFORM_MODE_INVERSE: u32;
    #[doc(hidden)]
    const DTYPE: c_int;
}

macro_rules! sort_key {
    ($t:ty, $dt:expr, $size:expr, $xf:expr, $w64:expr, $fwd:expr, $inv:expr) => {
        impl SortKey for $t {
            const KEY_SIZE: usize = $size;
            const NEEDS_TRANSFORM: bool = $xf;
            const IS_64BIT: bool = $w64;
            const TRANSFORM_MODE_FORWARD: u32 = $fwd;
            const TRANSFORM_MODE_INVERSE: u32 = $inv;
            const DTYPE: c_int = $dt;
        }
    };
}
sort_key!(u32, ffi::FS_U32, 4, false, false, 0, 0);
sort_key!(i32, ffi::FS_I32, 4, true, false, 0, 0);
sort_key!(f32, ffi::FS_F32, 4, true, false, 1, 2);
sort_key!(u64, ffi::FS_U64, 8, false, true, 0, 0);
sort_key!(i64, ffi::FS_I64, 8, true, true, 0, 0);
sort_key!(f64, ffi::FS_F64, 8, true, true, 1, 2);

/// forge-sort's error enum, with its Display strings (src/lib.rs:94-104).
#[derive(Debug)]
pub enum SortError {
    DeviceNotFound,
    ShaderCompilation(String),
    GpuExecution(String),
    LengthMismatch { keys: usize, values: usize },
}

impl fmt::Display for SortError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        match self {
            SortError::DeviceNotFound => write!(f, "no Metal GPU device found"),
            SortError::ShaderCompilation(m) => write!(f, "shader compilation failed: {m}"),
            SortError::GpuExecution(m) => write!(f, "GPU execution failed: {m}"),
            SortError::LengthMismatch { keys, values } => {
                write!(f, "length mismatch: keys={keys}, values={values}")
            }
        }
    }
}

impl std::error::Error for SortError {}

fn error_text(s: *const ffi::FsSorter) -> String {
    unsafe {
        let p = ffi::fs_last_error(s);
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

/// fs_status -> SortError: 1..4 are the four variants; timeouts, collective
/// failures, out-of-memory and bad arguments are GpuExecution(text).
fn check(rc: c_int, s: *const ffi::FsSorter) -> Result<(), SortError> {
    match rc {
        ffi::FS_OK => Ok(()),
        ffi::FS_E_DEVICE_NOT_FOUND => Err(SortError::DeviceNotFound),
        ffi::FS_E_KERNEL_IMAGE => Err(SortError::ShaderCompilation(error_text(s))),
        _ => Err(SortError::GpuExecution(error_text(s))),
    }
}

/// The library's buffer object, as given up by `SortBuffer::into_raw_parts`.
pub struct RawBuffer(NonNull<ffi::FsBuffer>);

/// A buffer the CPU and the GPU share (src/lib.rs:160-281).
pub struct SortBuffer<T: SortKey> {
    buf: NonNull<ffi::FsBuffer>,
    len: usize,
    capacity: usize,
    _t: PhantomData<T>,
}

unsafe impl<T: SortKey> Send for SortBuffer<T> {}

impl<T: SortKey> SortBuffer<T> {
    fn host(&self) -> *mut T {
        unsafe { ffi::fs_buffer_host(self.buf.as_ptr()) as *mut T }
    }

    pub fn len(&self) -> usize {
        self.len
    }

    pub fn is_empty(&self) -> bool {
        self.len == 0
    }

    pub fn capacity(&self) -> usize {
        self.capacity
    }

    /// All `capacity` elements for writing; then `set_len`.  The device copy
    /// is marked stale, so the next sort copies over what was written.
    pub fn as_mut_slice(&mut self) -> &mut [T] {
        let rc = unsafe { ffi::fs_buffer_host_write(self.buf.as_ptr()) };
        check(rc, std::ptr::null()).expect("SortBuffer host write");
        unsafe { std::slice::from_raw_parts_mut(self.host(), self.capacity) }
    }

    /// The first `len` elements (the sorted keys after a sort): waits for the
    /// sorts that touched the buffer and copies back what they changed.
    pub fn as_slice(&self) -> &[T] {
        let rc = unsafe { ffi::fs_buffer_host_read(self.buf.as_ptr()) };
        check(rc, std::ptr::null()).expect("SortBuffer host read");
        unsafe { std::slice::from_raw_parts(self.host(), self.len) }
    }

    /// Panics if `len > capacity`.
    pub fn set_len(&mut self, len: usize) {
        assert!(len <= self.capacity, "len {} exceeds capacity {}", len, self.capacity);
        self.len = len;
    }

    /// Panics if `data.len() > capacity`.
    pub fn copy_from_slice(&mut self, data: &[T]) {
        assert!(data.len() <= self.capacity, "data len {} exceeds capacity {}", data.len(), self.capacity);
        let dst = self.as_mut_slice();
        dst[..data.len()].copy_from_slice(data);
        self.len = data.len();
    }

    pub fn copy_to_slice(&self, dest: &mut [T]) {
        let n = self.len.min(dest.len());
        dest[..n].copy_from_slice(&self.as_slice()[..n]);
    }

    /// Device address of element 0 for other device code: the device copy is
    /// made current for `len` elements and counted as written.
    pub fn device_ptr(&self) -> *mut c_void {
        let bytes = (self.len * T::KEY_SIZE) as u64;
        let rc = unsafe { ffi::fs_buffer_device_use(self.buf.as_ptr(), bytes) };
        check(rc, std::ptr::null()).expect("SortBuffer device use");
        unsafe { ffi::fs_buffer_device(self.buf.as_ptr()) }
    }

    #[deprecated(note = "the buffer lives on a CUDA device: use device_ptr()")]
    pub fn metal_buffer(&self) -> *mut c_void {
        self.device_ptr()
    }

    /// Re-wrap a buffer object given up by `into_raw_parts`.
    pub fn from_raw_parts(buffer: RawBuffer, len: usize, capacity: usize) -> Self {
        assert!(len <= capacity, "len {len} exceeds capacity {capacity}");
        let bytes = unsafe { ffi::fs_buffer_bytes(buffer.0.as_ptr()) } as usize;
        assert!(capacity * T::KEY_SIZE <= bytes, "capacity exceeds the buffer's size");
        SortBuffer { buf: buffer.0, len, capacity, _t: PhantomData }
    }

    pub fn into_raw_parts(self) -> (RawBuffer, usize, usize) {
        let parts = (RawBuffer(self.buf), self.len, self.capacity);
        std::mem::forget(self);
        parts
    }
}

impl<T: SortKey> Drop for SortBuffer<T> {
    fn drop(&mut self) {
        unsafe {
            ffi::fs_buffer_destroy(self.buf.as_ptr());
        }
    }
}

/// GPU radix sort (src/lib.rs:132-3015): one CUDA device, one stream, a
/// grow-only scratch arena reused across calls and key types.
pub struct GpuSorter {
    h: NonNull<ffi::FsSorter>,
}

unsafe impl Send for GpuSorter {}

impl GpuSorter {
    /// Device 0 and a private stream (src/lib.rs:596).
    pub fn new() -> Result<Self, SortError> {
        Self::create(0, std::ptr::null_mut())
    }

    /// A caller's CUDA device ordinal and `cudaStream_t` (src/lib.rs:606,
    /// where a Metal device and command queue were passed).
    pub fn with_context(device: i32, stream: *mut c_void) -> Result<Self, SortError> {
        Self::create(device, stream)
    }

    fn create(device: i32, stream: *mut c_void) -> Result<Self, SortError> {
        let mut h = std::ptr::null_mut();
        check(unsafe { ffi::fs_create(device, stream, &mut h) }, std::ptr::null())?;
        Ok(GpuSorter { h: NonNull::new(h).ok_or(SortError::DeviceNotFound)? })
    }

    fn p(&self) -> *mut ffi::FsSorter {
        self.h.as_ptr()
    }

    /// Panics when the allocation fails, as the Metal crate's alloc_buffer
    /// did (src/metal_helpers.rs:194-202).
    pub fn alloc_sort_buffer<T: SortKey>(&self, capacity: usize) -> SortBuffer<T> {
        let mut b = std::ptr::null_mut();
        let bytes = (capacity.max(1) * T::KEY_SIZE) as u64;
        check(unsafe { ffi::fs_buffer_create(self.p(), bytes, &mut b) }, self.p()).expect("alloc_sort_buffer");
        SortBuffer { buf: NonNull::new(b).expect("alloc_sort_buffer"), len: 0, capacity, _t: PhantomData }
    }

    fn sort_buf<T: SortKey>(&mut self, buf: &SortBuffer<T>, sync: bool) -> Result<(), SortError> {
        if buf.len() <= 1 {
            return Ok(());
        }
        let rc = unsafe { ffi::fs_sort_buffer(self.p(), T::DTYPE, buf.buf.as_ptr(), buf.len() as u64, sync as c_int) };
        check(rc, self.p())
    }

    pub fn sort_buffer(&mut self, buf: &SortBuffer<u32>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }
    pub fn sort_i32_buffer(&mut self, buf: &SortBuffer<i32>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }
    pub fn sort_f32_buffer(&mut self, buf: &SortBuffer<f32>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }
    pub fn sort_u64_buffer(&mut self, buf: &SortBuffer<u64>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }
    pub fn sort_i64_buffer(&mut self, buf: &SortBuffer<i64>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }
    pub fn sort_f64_buffer(&mut self, buf: &SortBuffer<f64>) -> Result<(), SortError> {
        self.sort_buf(buf, true)
    }

    /// Enqueue an in-place sort of `buf` on `stream` (null: the sorter's own)
    /// and return (src/lib.rs:749-785); reading the buffer waits for it.
    pub fn encode_sort(&mut self, stream: *mut c_void, buf: &SortBuffer<u32>) -> Result<(), SortError> {
        if buf.len() <= 1 {
            return Ok(());
        }
        if !stream.is_null() {
            check(unsafe { ffi::fs_set_stream(self.p(), stream) }, self.p())?;
        }
        self.sort_buf(buf, false)
    }

    /// Wait for enqueued work and report device-side failures.
    pub fn synchronize(&mut self) -> Result<(), SortError> {
        check(unsafe { ffi::fs_synchronize(self.p()) }, self.p())
    }

    fn sort_host<T: SortKey>(&mut self, data: &mut [T]) -> Result<(), SortError> {
        if data.len() <= 1 {
            return Ok(());
        }
        let rc = unsafe { ffi::fs_host_sort_keys(self.p(), T::DTYPE, data.as_mut_ptr() as *mut c_void, data.len() as u64) };
        check(rc, self.p())
    }

    pub fn sort_u32(&mut self, data: &mut [u32]) -> Result<(), SortError> {
        self.sort_host(data)
    }
    pub fn sort_i32(&mut self, data: &mut [i32]) -> Result<(), SortError> {
        self.sort_host(data)
    }
    pub fn sort_f32(&mut self, data: &mut [f32]) -> Result<(), SortError> {
        self.sort_host(data)
    }
    pub fn sort_u64(&mut self, data: &mut [u64]) -> Result<(), SortError> {
        self.sort_host(data)
    }
    pub fn sort_i64(&mut self, data: &mut [i64]) -> Result<(), SortError> {
        self.sort_host(data)
    }
    pub fn sort_f64(&mut self, data: &mut [f64]) -> Result<(), SortError> {
        self.sort_host(data)
    }

    fn argsort_host<T: SortKey>(&mut self, data: &[T]) -> Result<Vec<u32>, SortError> {
        match data.len() {
            0 => return Ok(vec![]),
            1 => return Ok(vec![0]),
            _ => {}
        }
        let mut idx = vec![0u32; data.len()];
        let rc = unsafe {
            ffi::fs_host_argsort(self.p(), T::DTYPE, data.as_ptr() as *const c_void, idx.as_mut_ptr(),
                                 data.len() as u64)
        };
        check(rc, self.p())?;
        Ok(idx)
    }

    pub fn argsort_u32(&mut self, data: &[u32]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }
    pub fn argsort_i32(&mut self, data: &[i32]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }
    pub fn argsort_f32(&mut self, data: &[f32]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }
    pub fn argsort_u64(&mut self, data: &[u64]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }
    pub fn argsort_i64(&mut self, data: &[i64]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }
    pub fn argsort_f64(&mut self, data: &[f64]) -> Result<Vec<u32>, SortError> {
        self.argsort_host(data)
    }

    /// Length check first, then the n <= 1 short-cut (src/lib.rs:1928-1937).
    fn pairs_host<T: SortKey>(&mut self, keys: &mut [T], values: &mut [u32]) -> Result<(), SortError> {
        if keys.len() != values.len() {
            return Err(SortError::LengthMismatch { keys: keys.len(), values: values.len() });
        }
        if keys.len() <= 1 {
            return Ok(());
        }
        let rc = unsafe {
            ffi::fs_host_sort_pairs(self.p(), T::DTYPE, keys.as_mut_ptr() as *mut c_void, keys.len() as u64,
                                    values.as_mut_ptr(), values.len() as u64)
        };
        check(rc, self.p())
    }

    pub fn sort_pairs_u32(&mut self, keys: &mut [u32], values: &mut [u32]) -> Result<(), SortError> {
        self.pairs_host(keys, values)
    }
    pub fn sort_pairs_i32(&mut self, keys: &mut [i32], values: &mut [u32]) -> Result<(), SortError> {
        self.pairs_host(keys, values)
    }
    pub fn sort_pairs_f32(&mut self, keys: &mut [f32], values: &mut [u32]) -> Result<(), SortError> {
        self.pairs_host(keys, values)
    }
    pub fn sort_pairs_u64(&mut self, keys: &mut [u64], values: &mut [u32]) -> Result<(), SortError> {
        self.pairs_host(keys, values)
    }
    pub fn sort_pairs_i64(&mut self, keys: &mut [i64], values: &mut [u32]) -> Result<(), SortError> {
        self.pairs_host(keys, values)
    }

    /// Additive (not in the Metal crate): stable pairs sort of two
    /// SortBuffers on the device -- the 256M-pair configuration's path.
    pub fn sort_pairs_buffer<T: SortKey>(&mut self, keys: &SortBuffer<T>, values: &SortBuffer<u32>)
                                         -> Result<(), SortError> {
        if keys.len() != values.len() {
            return Err(SortError::LengthMismatch { keys: keys.len(), values: values.len() });
        }
        if keys.len() <= 1 {
            return Ok(());
        }
        let rc = unsafe {
            ffi::fs_sort_pairs_buffer(self.p(), T::DTYPE, keys.buf.as_ptr(), values.buf.as_ptr(), keys.len() as u64, 1)
        };
        check(rc, self.p())
    }
}

impl Drop for GpuSorter {
    fn drop(&mut self) {
        unsafe {
            ffi::fs_destroy(self.p());
        }
    }
}

/// Additive: the sample sort over several GPUs of one process (no
/// counterpart in the Metal crate).  Shard i lives on devices[i]; the output
/// pieces, concatenated in device order, are the sorted input.
pub struct MultiGpuSorter {
    mg: NonNull<ffi::FsMg>,
    devices: Vec<i32>,
}

/// One device allocation of a multi-GPU sort: `ptr` on devices[i], room for
/// `cap` keys, `len` of them in use.
#[derive(Clone, Copy, Debug)]
pub struct DeviceShard {
    pub ptr: *mut c_void,
    pub len: u64,
    pub cap: u64,
}

impl MultiGpuSorter {
    pub fn new(devices: &[i32]) -> Result<Self, SortError> {
        let mut mg = std::ptr::null_mut();
        let rc = unsafe { ffi::fs_mg_create(devices.as_ptr(), devices.len() as c_int, &mut mg) };
        check(rc, std::ptr::null())?;
        Ok(MultiGpuSorter { mg: NonNull::new(mg).ok_or(SortError::DeviceNotFound)?, devices: devices.to_vec() })
    }

    pub fn devices(&self) -> &[i32] {
        &self.devices
    }

    /// Sort the shards' keys across the GPUs; on return `out[i].len` holds
    /// the length of piece i.
    ///
    /// # Safety
    /// Every pointer must be device memory of the matching device with room
    /// for the stated number of keys of type T.
    pub unsafe fn sort_keys<T: SortKey>(&mut self, shards: &[DeviceShard], out: &mut [DeviceShard])
                                        -> Result<(), SortError> {
        let g = self.devices.len();
        assert!(shards.len() == g && out.len() == g, "one shard and one output per device");
        let sp: Vec<*mut c_void> = shards.iter().map(|s| s.ptr).collect();
        let sn: Vec<u64> = shards.iter().map(|s| s.len).collect();
        let op: Vec<*mut c_void> = out.iter().map(|s| s.ptr).collect();
        let oc: Vec<u64> = out.iter().map(|s| s.cap).collect();
        let mut on = vec![0u64; g];
        let rc = ffi::fs_mg_sort_keys(self.mg.as_ptr(), T::DTYPE, sp.as_ptr(), sn.as_ptr(), op.as_ptr(), oc.as_ptr(),
                                      on.as_mut_ptr());
        if rc != ffi::FS_OK {
            let p = ffi::fs_mg_last_error(self.mg.as_ptr());
            let text = if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() };
            return Err(SortError::GpuExecution(text));
        }
        for (o, n) in out.iter_mut().zip(on) {
            o.len = n;
        }
        Ok(())
    }

    /// # Safety
    /// As `sort_keys`, for u32 keys.
    pub unsafe fn sort_u32(&mut self, shards: &[DeviceShard], out: &mut [DeviceShard]) -> Result<(), SortError> {
        self.sort_keys::<u32>(shards, out)
    }

    /// # Safety
    /// As `sort_keys`, for u64 keys.
    pub unsafe fn sort_u64(&mut self, shards: &[DeviceShard], out: &mut [DeviceShard]) -> Result<(), SortError> {
        self.sort_keys::<u64>(shards, out)
    }
}

impl Drop for MultiGpuSorter {
    fn drop(&mut self) {
        unsafe {
            ffi::fs_mg_destroy(self.mg.as_ptr());
        }
    }
}

#[cfg(test)]
mod tests {
    use super::*;

    // the reference's own unit test of the Display strings (src/lib.rs:3034-3049)
    #[test]
    fn sort_error_display() {
        assert_eq!(SortError::DeviceNotFound.to_string(), "no Metal GPU device found");
        assert_eq!(SortError::ShaderCompilation("test".into()).to_string(), "shader compilation failed: test");
        assert_eq!(SortError::GpuExecution("timeout".into()).to_string(), "GPU execution failed: timeout");
        assert_eq!(SortError::LengthMismatch { keys: 10, values: 5 }.to_string(), "length mismatch: keys=10, values=5");
    }

    #[test]
    fn sort_u32_basic() {
        let mut s = match GpuSorter::new() {
            Ok(s) => s,
            Err(SortError::DeviceNotFound) => return,
            Err(e) => panic!("{e}"),
        };
        let mut v = vec![30u32, 10, 20, 5, 1];
        s.sort_u32(&mut v).unwrap();
        assert_eq!(v, vec![1, 5, 10, 20, 30]);
        assert_eq!(s.argsort_u32(&[30, 10, 20]).unwrap(), vec![1, 2, 0]);
        let mut buf = s.alloc_sort_buffer::<f32>(4);
        buf.copy_from_slice(&[2.5, -1.0, 0.0, -0.0]);
        s.sort_f32_buffer(&buf).unwrap();
        let got: Vec<u32> = buf.as_slice().iter().map(|x| x.to_bits()).collect();
        assert_eq!(got, vec![(-1.0f32).to_bits(), (-0.0f32).to_bits(), 0.0f32.to_bits(), 2.5f32.to_bits()]);
    }
}
