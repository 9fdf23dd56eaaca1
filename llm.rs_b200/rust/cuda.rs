//! `CudaBackend`: the reference's `trait Backend` (src/backend.rs:15-40) on the
//! B200 library `libllmrs_cuda.so` (`src/backend/cuda.rs` in the maintainer's
//! tree, with `ffi.rs` beside it as `src/backend/cuda/ffi.rs`).
//!
//! UNVERIFIED: this image has no Rust toolchain, so this file has never been
//! compiled; it is written against the reference's types as they stand
//! (`Tensor`, `Storage`, `Shape`, `Device` in src/core/tensor.rs,
//! src/core/shape.rs and src/backend.rs) plus the additions listed in the
//! "storage additions" block at the end of this file.
//!
//! Two routes, as in the C header:
//! * per op: every trait method is one library call on device f32 buffers;
//!   results are new device tensors (the reference's ops return new, allocated
//!   tensors; in-place ops mutate through `Arc::get_mut` and panic when the
//!   storage is shared, src/backend/cpu.rs:278-284);
//! * whole model: `CudaModel` keeps weights and the KV cache on the device and
//!   runs a decode step as one CUDA graph (replaces `LlamaModel::forward` for a
//!   1-token chunk, src/core/model.rs:17-49, and the token loop of
//!   src/main.rs:128-190).  This is the fast route.
use std::os::raw::{c_int, c_void};
use std::sync::{Arc, OnceLock};

use super::ffi::{self, check};
use crate::backend::{Backend, Device};
use crate::core::shape::Shape;
use crate::core::tensor::{Storage, Tensor};

// ------------------------------------------------------------------ context
/// The process-wide library context on GPU 0 (the reference's OpenCL backend
/// keeps one global queue the same way).  Set LLMRS_DEVICE to pick a GPU.
struct Ctx(*mut ffi::llmrs_ctx);
unsafe impl Send for Ctx {}
unsafe impl Sync for Ctx {}

static CTX: OnceLock<Ctx> = OnceLock::new();

pub fn ctx() -> *mut ffi::llmrs_ctx {
    CTX.get_or_init(|| {
        let device = std::env::var("LLMRS_DEVICE").ok().and_then(|v| v.parse().ok()).unwrap_or(0);
        let mut c = std::ptr::null_mut();
        check(unsafe { ffi::llmrs_ctx_create(device, &mut c) });
        Ctx(c)
    })
    .0
}

// ---------------------------------------------------------- device buffers
/// Device memory owned by a tensor; freed when the last `Arc<Storage>` goes.
#[derive(Debug)]
pub struct DeviceBuf {
    pub ptr: *mut c_void,
    pub bytes: usize,
}
unsafe impl Send for DeviceBuf {}
unsafe impl Sync for DeviceBuf {}

impl DeviceBuf {
    pub fn alloc(bytes: usize) -> Self {
        let mut ptr = std::ptr::null_mut();
        check(unsafe { ffi::llmrs_malloc(ctx(), bytes.max(16), &mut ptr) });
        DeviceBuf { ptr, bytes }
    }
    pub fn upload<T>(host: &[T]) -> Self {
        let bytes = std::mem::size_of_val(host);
        let b = Self::alloc(bytes);
        check(unsafe { ffi::llmrs_h2d(ctx(), b.ptr, host.as_ptr() as *const c_void, bytes) });
        b
    }
    pub fn download_f32(&self, n: usize) -> Vec<f32> {
        let mut v = vec![0.0f32; n];
        check(unsafe { ffi::llmrs_d2h(ctx(), v.as_mut_ptr() as *mut c_void, self.ptr, n * 4) });
        v
    }
}

impl Drop for DeviceBuf {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe { ffi::llmrs_free(ctx(), self.ptr) };
        }
    }
}

fn dims2(t: &Tensor) -> (usize, usize) {
    let d = t.shape().dims();
    match d.len() {
        0 => (0, 0),
        1 => (1, d[0]),
        _ => (d[..d.len() - 1].iter().product(), d[d.len() - 1]),
    }
}

/// Device pointer of an f32 tensor (panics for other storage, like the
/// reference's CPU backend does for storage it cannot read).
fn dptr(t: &Tensor) -> *const f32 {
    match &*t.storage {
        Storage::Cuda(b) => b.ptr as *const f32,
        _ => panic!("CudaBackend requires Cuda storage"),
    }
}

fn dptr_mut(t: &mut Tensor) -> *mut f32 {
    match Arc::get_mut(&mut t.storage) {
        Some(Storage::Cuda(b)) => b.ptr as *mut f32,
        Some(_) => panic!("CudaBackend requires Cuda storage"),
        None => panic!("Cannot mutate: storage is shared"),
    }
}

fn new_device_tensor(shape: Shape) -> (Tensor, *mut f32) {
    let b = DeviceBuf::alloc(shape.num_elements() * 4);
    let p = b.ptr as *mut f32;
    (Tensor::from_storage(Storage::Cuda(b), shape, Device::Cuda), p)
}

fn ci(v: usize) -> c_int {
    c_int::try_from(v).expect("dimension exceeds the C ABI's int range")
}

// ------------------------------------------------------------------ backend
pub struct CudaBackend;

impl CudaBackend {
    pub fn new() -> Self {
        let _ = ctx();
        CudaBackend
    }
}

impl Default for CudaBackend {
    fn default() -> Self {
        Self::new()
    }
}

impl Backend for CudaBackend {
    fn device(&self) -> Device {
        Device::Cuda
    }

    fn name(&self) -> &str {
        "Cuda (B200, sm_100a)"
    }

    /// A[m,k] @ B[k,n] (src/backend/cpu.rs:157-224).
    fn matmul(&self, a: &Tensor, b: &Tensor) -> Tensor {
        let (m, k) = (a.shape().dims()[0], a.shape().dims()[1]);
        let (k2, n) = (b.shape().dims()[0], b.shape().dims()[1]);
        assert_eq!(k, k2, "MatMul Dimension mismatch");
        let (out, c) = new_device_tensor(Shape::new(vec![m, n]));
        check(unsafe { ffi::llmrs_matmul(ctx(), dptr(a), dptr(b), c, ci(m), ci(k), ci(n)) });
        out
    }

    /// A[m,k] @ W[n,k]^T (src/backend/cpu.rs:31-111): W in the reference's
    /// planar Q4_0 (nibbles + f32 block scales, as `quantize_q4` made them),
    /// Q8_0 codes, or f32.  m == 1 is the batch-1 GEMV with the fused Q8_0
    /// activation quantiser; m >= 8 runs on the tensor cores.
    fn matmul_transposed(&self, a: &Tensor, b: &Tensor) -> Tensor {
        let (m, k) = (a.shape().dims()[0], a.shape().dims()[1]);
        let n = b.shape().dims()[0];
        let (out, c) = new_device_tensor(Shape::new(vec![m, n]));
        let rc = match &*b.storage {
            Storage::CudaQ4 { qs, scales, scale_dtype } => unsafe {
                ffi::llmrs_matmul_transposed_q4(ctx(), dptr(a), qs.ptr as *const u8, scales.ptr, *scale_dtype, c,
                                                ci(m), ci(k), ci(n))
            },
            Storage::CudaQ8 { codes, scales, scale_dtype } => unsafe {
                ffi::llmrs_matmul_transposed_q8(ctx(), dptr(a), codes.ptr as *const i8, scales.ptr, *scale_dtype,
                                                c, ci(m), ci(k), ci(n))
            },
            Storage::Cuda(w) => unsafe {
                assert_eq!(b.shape().dims()[1], k, "MatMul Transposed mismatch");
                ffi::llmrs_matmul_transposed_f32(ctx(), dptr(a), w.ptr as *const f32, c, ci(m), ci(k), ci(n))
            },
            _ => panic!("Unsupported storage type for B in matmul_transposed"),
        };
        check(rc);
        out
    }

    /// A[m,cols] @ S[rows,cols]^T with S a host slice (src/backend/cpu.rs:230-269;
    /// the reference's KV-cache attention passes the cache this way).  The slice
    /// is copied to the device for the call.
    fn matmul_slice(&self, a: &Tensor, other_data: &[f32], rows: usize, cols: usize) -> Tensor {
        let (m, k) = (a.shape().dims()[0], a.shape().dims()[1]);
        assert_eq!(k, cols, "MatMul Slice mismatch");
        assert!(other_data.len() >= rows * cols, "MatMul Slice: slice too short");
        let other = DeviceBuf::upload(&other_data[..rows * cols]);
        let (out, c) = new_device_tensor(Shape::new(vec![m, rows]));
        check(unsafe {
            ffi::llmrs_matmul_slice(ctx(), dptr(a), other.ptr as *const f32, c, ci(m), ci(rows), ci(cols))
        });
        out
    }

    /// a += b (src/backend/cpu.rs:274-296)
    fn add_assign(&self, a: &mut Tensor, b: &Tensor) {
        if a.shape() != b.shape() {
            panic!("Shape mismatch in add_assign");
        }
        let n = a.shape().num_elements();
        let bp = dptr(b);
        let ap = dptr_mut(a);
        check(unsafe { ffi::llmrs_add_assign(ctx(), ap, bp, n) });
    }

    /// gate = silu(gate) * up (src/backend/cpu.rs:298-324)
    fn silu_mul(&self, gate: &mut Tensor, up: &Tensor) {
        if gate.shape() != up.shape() {
            panic!("Shape mismatch in silu_mul");
        }
        let n = gate.shape().num_elements();
        let up_p = dptr(up);
        let gp = dptr_mut(gate);
        check(unsafe { ffi::llmrs_silu_mul(ctx(), gp, up_p, n) });
    }

    /// Rotate-half RoPE of rows of the last dimension at positions
    /// start_pos + row (src/backend/cpu.rs:326-357; theta 500000 as there).
    fn rope_inplace(&self, x: &mut Tensor, start_pos: usize) {
        let (rows, head_dim) = dims2(x);
        let xp = dptr_mut(x);
        check(unsafe { ffi::llmrs_rope_inplace(ctx(), xp, ci(rows), ci(head_dim), ci(start_pos), 500_000.0) });
    }

    /// RMSNorm over the last dimension (src/backend/cpu.rs:359-393)
    fn rms_norm(&self, x: &Tensor, weight: &Tensor, eps: f32) -> Tensor {
        let (rows, cols) = dims2(x);
        assert_eq!(weight.shape().num_elements(), cols, "RMSNorm weight size mismatch");
        let (out, y) = new_device_tensor(x.shape().clone());
        check(unsafe { ffi::llmrs_rms_norm(ctx(), dptr(x), dptr(weight), y, ci(rows), ci(cols), eps) });
        out
    }

    /// Softmax over the last dimension (src/backend/cpu.rs:395-423)
    fn softmax(&self, x: &Tensor) -> Tensor {
        let (rows, cols) = dims2(x);
        let (out, y) = new_device_tensor(x.shape().clone());
        check(unsafe { ffi::llmrs_softmax(ctx(), dptr(x), y, ci(rows), ci(cols)) });
        out
    }

    /// x * value (src/backend/cpu.rs:425-435)
    fn scale(&self, x: &Tensor, value: f32) -> Tensor {
        let n = x.shape().num_elements();
        let (out, y) = new_device_tensor(x.shape().clone());
        check(unsafe { ffi::llmrs_scale(ctx(), dptr(x), y, n, value) });
        out
    }

    /// A new tensor with the same contents (src/backend/cpu.rs:437-446)
    fn copy_from(&self, tensor: &Tensor) -> Tensor {
        let n = tensor.shape().num_elements();
        let (out, y) = new_device_tensor(tensor.shape().clone());
        check(unsafe { ffi::llmrs_copy_from(ctx(), dptr(tensor), y, n) });
        out
    }
}

// ------------------------------------------------------------- whole model
/// Device-resident model: weights in the reference's Q4_0 (or Q8_0) block
/// layout, the KV cache and the decode step's CUDA graph, all on the GPU.
pub struct CudaModel {
    h: *mut ffi::llmrs_model,
    pub cfg: ffi::llmrs_config,
}
unsafe impl Send for CudaModel {}

impl CudaModel {
    /// `cfg` from the reference's LlamaConfig (src/core/config.rs): max_seq is
    /// the KV capacity (the reference hard-codes 2048, src/core/loader.rs:162-166).
    pub fn new(cfg: ffi::llmrs_config) -> Self {
        let mut h = std::ptr::null_mut();
        check(unsafe { ffi::llmrs_model_create(ctx(), &cfg, &mut h) });
        CudaModel { h, cfg }
    }

    /// One checkpoint tensor in the loader's layout (src/core/loader.rs:25-198):
    /// bf16 (`LLMRS_BF16`) or f32 values, quantised on the device exactly like
    /// `Tensor::quantize_q4`; `which` = `ffi::LLMRS_W_*`; norms and the embedding
    /// stay f32.  q/k/v rows keep native GQA, gate/up may come separately
    /// (`LLMRS_W_GATE`, `LLMRS_W_UP`), a tied LM head follows the embedding.
    pub fn load_weight(&mut self, layer: usize, which: c_int, data: &[u8], dtype: c_int) {
        check(unsafe {
            ffi::llmrs_model_load_weight(self.h, ci(layer), which, data.as_ptr() as *const c_void, dtype)
        });
    }

    /// A tensor already quantised on the host (planar nibbles + f32 scales as
    /// `quantize_q4` returns them, `Storage::CpuQ4`).
    pub fn set_weight_q4(&mut self, layer: usize, which: c_int, codes: &[u8], scales: &[f32]) {
        check(unsafe {
            ffi::llmrs_model_set_weight(self.h, ci(layer), which, codes.as_ptr() as *const c_void, scales.as_ptr())
        });
    }

    /// An f32 tensor (norm weights, embedding).
    pub fn set_weight_f32(&mut self, layer: usize, which: c_int, values: &[f32]) {
        check(unsafe {
            ffi::llmrs_model_set_weight(self.h, ci(layer), which, values.as_ptr() as *const c_void,
                                        std::ptr::null())
        });
    }

    /// Prompt chunk at positions start_pos.. (prefill on the tensor cores for
    /// 8 or more tokens); returns the last row's logits and greedy token.
    pub fn prefill(&mut self, ids: &[u32], start_pos: usize) -> (Vec<f32>, u32) {
        let ids: Vec<c_int> = ids.iter().map(|&t| t as c_int).collect();
        let mut logits = vec![0.0f32; self.cfg.vocab as usize];
        let mut arg: c_int = 0;
        check(unsafe {
            ffi::llmrs_prefill(self.h, ids.as_ptr(), ci(ids.len()), ci(start_pos), logits.as_mut_ptr(), &mut arg)
        });
        (logits, arg as u32)
    }

    /// One decode step of `token` at `pos` (src/main.rs:128-190 for one token):
    /// greedy token out; logits copied back only when asked for (sampling can
    /// stay on the device with `sample`).
    pub fn decode_step(&mut self, token: u32, pos: usize, want_logits: bool) -> (Option<Vec<f32>>, u32) {
        let mut arg: c_int = 0;
        if want_logits {
            let mut logits = vec![0.0f32; self.cfg.vocab as usize];
            check(unsafe {
                ffi::llmrs_decode_step(self.h, token as c_int, ci(pos), logits.as_mut_ptr(), &mut arg)
            });
            (Some(logits), arg as u32)
        } else {
            check(unsafe { ffi::llmrs_decode_step(self.h, token as c_int, ci(pos), std::ptr::null_mut(), &mut arg) });
            (None, arg as u32)
        }
    }

    /// src/main.rs:192-305 on the device over the last step's logits: the
    /// caller's recent ids (the penalty window) and its uniform draw `u`
    /// (`rng.random::<f32>()` in the reference).
    pub fn sample(&mut self, recent: &[u32], repeat_penalty: f32, temperature: f32, top_p: f32, u: f32) -> u32 {
        let recent: Vec<c_int> = recent.iter().map(|&t| t as c_int).collect();
        let mut tok: c_int = 0;
        check(unsafe {
            ffi::llmrs_model_sample(self.h, recent.as_ptr(), ci(recent.len()), repeat_penalty, temperature, top_p,
                                    u, &mut tok)
        });
        tok as u32
    }
}

impl Drop for CudaModel {
    fn drop(&mut self) {
        if !self.h.is_null() {
            unsafe { ffi::llmrs_model_destroy(self.h) };
        }
    }
}

// ------------------------------------------------------ storage additions
// The reference's types gain these members (shown here, not compiled here):
//
// src/backend.rs, `enum Device`:            Cuda,
//
// src/core/tensor.rs, `enum Storage`:
//     Cuda(crate::backend::cuda::DeviceBuf),
//     CudaQ4 { qs: DeviceBuf, scales: DeviceBuf, scale_dtype: i32 },
//     CudaQ8 { codes: DeviceBuf, scales: DeviceBuf, scale_dtype: i32 },
//
// src/core/tensor.rs, `Tensor::backend()`:  Device::Cuda => Box::new(CudaBackend::new()),
//
// src/core/tensor.rs, `Tensor::to_device`, three new arms (below as a helper).

/// The `to_device` arms for the Cuda device: host f32 -> device, host Q4
/// (nibbles + f32 scales) -> device, device -> host f32.
pub fn to_device_cuda(t: &Tensor, target: Device) -> Option<Tensor> {
    match (&*t.storage, target) {
        (Storage::Cpu(v), Device::Cuda) => Some(Tensor::from_storage(
            Storage::Cuda(DeviceBuf::upload(v)), t.shape().clone(), Device::Cuda)),
        (Storage::CpuQ4 { data, scales }, Device::Cuda) => Some(Tensor::from_storage(
            Storage::CudaQ4 { qs: DeviceBuf::upload(data), scales: DeviceBuf::upload(scales),
                              scale_dtype: ffi::LLMRS_F32 },
            t.shape().clone(), Device::Cuda)),
        (Storage::Cuda(b), Device::Cpu) => {
            let n = t.shape().num_elements();
            Some(Tensor::new(b.download_f32(n), t.shape().clone()))
        }
        _ => None,
    }
}
