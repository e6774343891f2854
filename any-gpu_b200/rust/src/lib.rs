//! any-gpu's `GpuDevice` API on B200 (sm_100a): a drop-in for the reference
//! crate's `use any_gpu::{GpuDevice, GpuBuffer}` whose every op runs in
//! libagpu.so, the hand-written tcgen05 / TMA kernels behind `include/agpu.h`.
//!
//! ```no_run
//! use any_gpu::GpuDevice;
//! let dev = GpuDevice::gpu()?;
//! let a = dev.upload(&[1.0, 2.0, 3.0, 4.0]);
//! let b = dev.upload(&[5.0, 6.0, 7.0, 8.0]);
//! let c = dev.matmul(&a, &b, 2, 2, 2)?;          // (m, n, k), as the reference
//! assert_eq!(dev.read(&c)?, vec![19.0, 22.0, 43.0, 50.0]);
//! # Ok::<(), anyhow::Error>(())
//! ```

mod device;
pub mod ffi;

pub use device::{AgpuError, GpuBuffer, GpuDevice, Precision};
