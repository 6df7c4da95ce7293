// SPDX-License-Identifier: MIT OR Apache-2.0
//
// UNVERIFIED (see Cargo.toml): never compiled here. The sl-ir / sl-device
// items used are the ones docs/ARCH-0004 (Value, Op, DType, ValueRole,
// TensorEncoding) and docs/ARCH-0007 section 3.1 (Device, BufferRef,
// DeviceError) define; `Shape::dims()` is assumed to expose the `Vec<Dim>`.

//! [`CudaDevice`]: a [`sl_device::Device`] over `libslc.so`, the B200
//! (sm_100a) backend whose C ABI is `include/starlight_cuda.h` of the
//! starlight_b200 checkout.
//!
//! Every trait method is one call into the library, which repeats
//! `CpuDevice`'s validation (`validate_call`, `validate_port`,
//! `check_disjoint`, then each operator's geometry checks) before anything is
//! enqueued and returns the same `DeviceError` variants. `dispatch` converts
//! its arguments into fixed-size stack arrays (at most four input ports and
//! one output port, as every `sl_ir::Op` has), so it allocates nothing.

mod ffi;

use core::ffi::{c_int, CStr};

use sl_device::{BufferRef, Device, DeviceError};
use sl_ir::{BufferId, DType, Dim, Op, OpCode, QuantizationFormat, RopeVariant, TensorEncoding, Value,
            ValueRole};

pub use ffi::SlcCapabilities;

/// One CUDA device (one GPU, one stream) behind the `sl_device::Device` trait.
pub struct CudaDevice {
    raw: *mut ffi::SlcDevice,
}

// The library serialises every call on a device; the handle may move
// between threads (Device: Send).
unsafe impl Send for CudaDevice {}

impl CudaDevice {
    /// Creates the device for GPU `ordinal` (its stream and workspace).
    pub fn new(ordinal: i32) -> Result<Self, DeviceError> {
        let mut raw = core::ptr::null_mut();
        let rc = unsafe { ffi::slc_device_create(ordinal, &mut raw) };
        if rc != ffi::SLC_OK || raw.is_null() {
            return Err(DeviceError::Execution("cuda device creation failed"));
        }
        Ok(Self { raw })
    }

    /// The `DeviceCapabilities` the runtime declares for this backend.
    pub fn capabilities(&self) -> Result<SlcCapabilities, DeviceError> {
        let mut caps = SlcCapabilities::default();
        self.check(unsafe { ffi::slc_get_capabilities(self.raw, &mut caps) })?;
        Ok(caps)
    }

    /// Names `scales` as the scale buffer of the quantized payload `codes`
    /// (EXTENSION: the quantized `Param` binding the reference lacks).
    pub fn bind_quant(&mut self, codes: BufferId, scales: BufferId, format: QuantizationFormat,
                      group_size: u32) -> Result<(), DeviceError> {
        let f = match format { QuantizationFormat::Int4 => 0, QuantizationFormat::Int8 => 1 };
        self.check(unsafe { ffi::slc_bind_quant(self.raw, codes.0, scales.0, f, group_size) })
    }

    /// EXTENSION: record commands and replay repeated segments as CUDA graphs.
    pub fn set_capture(&mut self, enabled: bool) -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_set_capture(self.raw, enabled as c_int) })
    }

    /// EXTENSION: joins tensor-parallel rank `rank` of `world` (collective;
    /// `unique_id` from [`CudaDevice::comm_unique_id`] on rank 0).
    pub fn comm_init(&mut self, unique_id: &[u8; 128], rank: i32, world: i32)
                     -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_comm_init(self.raw, unique_id.as_ptr(), rank, world) })
    }

    pub fn comm_unique_id() -> Result<[u8; 128], DeviceError> {
        let mut id = [0u8; 128];
        match unsafe { ffi::slc_comm_unique_id(id.as_mut_ptr()) } {
            ffi::SLC_OK => Ok(id),
            _ => Err(DeviceError::Execution("NCCL unique id")),
        }
    }

    /// EXTENSION: drops the communicator without the other ranks (a peer
    /// left between steps); later collectives fail instead of waiting.
    pub fn comm_abort(&mut self) -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_comm_abort(self.raw) })
    }

    fn check(&self, rc: c_int) -> Result<(), DeviceError> {
        if rc == ffi::SLC_OK {
            return Ok(());
        }
        let mut e = ffi::SlcError { status: 0, buffer: 0, offset: 0, len: 0, requested: 0,
                                    opcode: 0, message: core::ptr::null() };
        unsafe { ffi::slc_last_error(self.raw, &mut e) };
        let msg: &'static str = if e.message.is_null() {
            "libslc error"
        } else {
            // Static strings of the library: valid for the life of the process.
            unsafe { CStr::from_ptr(e.message) }.to_str().unwrap_or("libslc error")
        };
        Err(match rc {
            ffi::SLC_ERR_OUT_OF_MEMORY => DeviceError::OutOfMemory { requested: e.requested as usize },
            ffi::SLC_ERR_INVALID_BUFFER => DeviceError::InvalidBuffer(BufferId(e.buffer)),
            ffi::SLC_ERR_INVALID_RANGE => DeviceError::InvalidRange {
                buffer: BufferId(e.buffer),
                offset: e.offset as usize,
                len: e.len as usize,
            },
            ffi::SLC_ERR_UNSUPPORTED_OP => match opcode_from_u16(e.opcode as u16) {
                Some(code) => DeviceError::UnsupportedOp(code),
                None => DeviceError::Execution(msg),
            },
            ffi::SLC_ERR_SHAPE_OVERFLOW => DeviceError::ShapeOverflow,
            ffi::SLC_ERR_UNIMPLEMENTED => DeviceError::Unimplemented(msg),
            _ => DeviceError::Execution(msg),
        })
    }
}

impl Drop for CudaDevice {
    fn drop(&mut self) {
        unsafe { ffi::slc_device_destroy(self.raw) }
    }
}

// ---- conversions (declaration orders are ABI, docs/ARCH-0004) -------------------

fn opcode_from_u16(code: u16) -> Option<OpCode> {
    use OpCode::*;
    const ALL: [OpCode; 18] = [MatMulNT, MatMulNN, Softmax, SoftmaxCausal, RmsNorm, Rope, Silu, Mul,
                               Add, Scale, Gather, LastToken, KvAppend, SplitHeads, MergeHeads,
                               CausalAttention, SwiGlu, RmsNormMatMul];
    ALL.get(code as usize).copied()
}

fn to_slc_op(op: &Op) -> ffi::SlcOp {
    let mut o = ffi::SlcOp { code: op.code() as u16, ..Default::default() };
    match *op {
        Op::RmsNorm { eps } | Op::RmsNormMatMul { eps } => o.eps = eps,
        Op::Rope { variant, theta } => {
            o.rope_variant = match variant { RopeVariant::Neox => 0, RopeVariant::GptJ => 1 };
            o.theta = theta;
        }
        Op::Scale { factor } => o.factor = factor,
        Op::KvAppend { layer } => o.layer = layer,
        Op::SplitHeads { heads, head_dim } | Op::MergeHeads { heads, head_dim } => {
            o.heads = heads;
            o.head_dim = head_dim;
        }
        Op::CausalAttention { layer, heads, kv_heads, head_dim, scale } => {
            o.layer = layer;
            o.heads = heads;
            o.kv_heads = kv_heads;
            o.head_dim = head_dim;
            o.scale = scale;
        }
        _ => {}
    }
    o
}

fn to_slc_value(v: &Value) -> Result<ffi::SlcValue, DeviceError> {
    let dims = v.shape.dims();
    if dims.len() > ffi::SLC_MAX_RANK {
        return Err(DeviceError::ShapeOverflow);
    }
    let mut out = ffi::SlcValue {
        dtype: match v.dtype {
            DType::F32 => 0, DType::F16 => 1, DType::BF16 => 2, DType::U32 => 3,
            DType::I32 => 4, DType::U8 => 5, DType::I8 => 6,
        },
        role: match v.role {
            ValueRole::Input => 0, ValueRole::Scalar => 1, ValueRole::Output => 2,
            ValueRole::Param => 3, ValueRole::State => 4, ValueRole::Temp => 5,
        },
        rank: dims.len() as u32,
        ..Default::default()
    };
    for (i, d) in dims.iter().enumerate() {
        out.dims[i] = match d {
            Dim::Const(n) => *n,
            // A CommandBuffer holds no symbolic dims (docs/ARCH-0004).
            Dim::Sym(_) => return Err(DeviceError::Execution("symbolic dimension in a command")),
        };
    }
    match &v.encoding {
        TensorEncoding::Dense => out.encoding = ffi::SLC_ENC_DENSE,
        TensorEncoding::GroupwiseQuantized { format, group_size } => {
            out.encoding = ffi::SLC_ENC_GROUPWISE;
            out.quant_format = match format { QuantizationFormat::Int4 => 0, QuantizationFormat::Int8 => 1 };
            out.group_size = *group_size;
        }
        // Rejected by the library with Unimplemented, as the reference requires.
        TensorEncoding::OpaqueQuantized { .. } => out.encoding = ffi::SLC_ENC_OPAQUE,
    }
    Ok(out)
}

fn to_slc_ref(r: &BufferRef) -> ffi::SlcBufferRef {
    ffi::SlcBufferRef { buffer: r.buffer.0, reserved: 0, offset: r.offset as u64, len: r.len as u64 }
}

impl Device for CudaDevice {
    fn allocate_f32(&mut self, elements: usize, align: usize) -> Result<BufferId, DeviceError> {
        let mut b = 0u32;
        self.check(unsafe { ffi::slc_allocate_f32(self.raw, elements as u64, align as u64, &mut b) })?;
        Ok(BufferId(b))
    }

    fn allocate_u32(&mut self, elements: usize, align: usize) -> Result<BufferId, DeviceError> {
        let mut b = 0u32;
        self.check(unsafe { ffi::slc_allocate_u32(self.raw, elements as u64, align as u64, &mut b) })?;
        Ok(BufferId(b))
    }

    fn upload_f32(&mut self, buffer: BufferId, data: &[f32]) -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_upload_f32(self.raw, buffer.0, data.as_ptr(), data.len() as u64) })
    }

    fn upload_u32(&mut self, buffer: BufferId, data: &[u32]) -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_upload_u32(self.raw, buffer.0, data.as_ptr(), data.len() as u64) })
    }

    fn download_f32(&mut self, buffer: BufferId, out: &mut [f32]) -> Result<(), DeviceError> {
        self.check(unsafe {
            ffi::slc_download_f32(self.raw, buffer.0, out.as_mut_ptr(), out.len() as u64)
        })
    }

    fn download_u32(&mut self, buffer: BufferId, out: &mut [u32]) -> Result<(), DeviceError> {
        self.check(unsafe {
            ffi::slc_download_u32(self.raw, buffer.0, out.as_mut_ptr(), out.len() as u64)
        })
    }

    fn dispatch(
        &mut self,
        op: &Op,
        inputs: &[BufferRef],
        input_values: &[&Value],
        outputs: &[BufferRef],
        output_values: &[&Value],
        scalars: &[u32],
    ) -> Result<(), DeviceError> {
        // The C ABI takes one count per side, so the first checks of
        // CpuDevice's validate_call (device.rs:232-244, same order and
        // messages) happen here; the library repeats the rest.
        if inputs.len() != input_values.len() {
            return Err(DeviceError::Execution("inputs and input_values have different lengths"));
        }
        if outputs.len() != output_values.len() {
            return Err(DeviceError::Execution("outputs and output_values have different lengths"));
        }
        if inputs.len() > 4 || outputs.len() > 1 {
            return Err(DeviceError::Execution("too many command ports"));
        }
        let mut ir = [ffi::SlcBufferRef::default(); 4];
        let mut iv = [ffi::SlcValue::default(); 4];
        let mut or = [ffi::SlcBufferRef::default(); 1];
        let mut ov = [ffi::SlcValue::default(); 1];
        for (i, r) in inputs.iter().enumerate() { ir[i] = to_slc_ref(r); }
        for (i, v) in input_values.iter().enumerate() { iv[i] = to_slc_value(v)?; }
        for (i, r) in outputs.iter().enumerate() { or[i] = to_slc_ref(r); }
        for (i, v) in output_values.iter().enumerate() { ov[i] = to_slc_value(v)?; }
        let o = to_slc_op(op);
        self.check(unsafe {
            ffi::slc_dispatch(self.raw, &o, ir.as_ptr(), iv.as_ptr(), inputs.len() as u64,
                              or.as_ptr(), ov.as_ptr(), outputs.len() as u64, scalars.as_ptr(),
                              scalars.len() as u64)
        })
    }

    fn synchronize(&mut self) -> Result<(), DeviceError> {
        self.check(unsafe { ffi::slc_synchronize(self.raw) })
    }
}
