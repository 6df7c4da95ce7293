// UNVERIFIED (see Cargo.toml): the #[repr(C)] mirror of include/starlight_cuda.h.
// Field order, widths and discriminants follow the header one to one.

use core::ffi::{c_char, c_int, c_void};

pub const SLC_MAX_RANK: usize = 8;

pub const SLC_OK: c_int = 0;
pub const SLC_ERR_OUT_OF_MEMORY: c_int = 1;
pub const SLC_ERR_INVALID_BUFFER: c_int = 2;
pub const SLC_ERR_INVALID_RANGE: c_int = 3;
pub const SLC_ERR_UNSUPPORTED_OP: c_int = 4;
pub const SLC_ERR_SHAPE_OVERFLOW: c_int = 5;
pub const SLC_ERR_EXECUTION: c_int = 6;
pub const SLC_ERR_UNIMPLEMENTED: c_int = 7;

pub const SLC_ENC_DENSE: u32 = 0;
pub const SLC_ENC_GROUPWISE: u32 = 1;
pub const SLC_ENC_OPAQUE: u32 = 2;

/// Last error of a device; `message` is a static string of the library.
#[repr(C)]
pub struct SlcError {
    pub status: i32,
    pub buffer: u32,
    pub offset: u64,
    pub len: u64,
    pub requested: u64,
    pub opcode: u32,
    pub message: *const c_char,
}

/// `sl_ir::Value` with constant dims.
#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct SlcValue {
    pub dtype: u32,
    pub role: u32,
    pub rank: u32,
    pub dims: [u32; SLC_MAX_RANK],
    pub encoding: u32,
    pub quant_format: u32,
    pub group_size: u32,
}

/// `sl_device::BufferRef` (offset and len in elements).
#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct SlcBufferRef {
    pub buffer: u32,
    pub reserved: u32,
    pub offset: u64,
    pub len: u64,
}

/// `sl_ir::Op`: the opcode and its variant's attributes.
#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct SlcOp {
    pub code: u16,
    pub rope_variant: u16,
    pub layer: u32,
    pub heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub eps: f32,
    pub theta: f32,
    pub scale: f32,
    pub factor: f32,
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct SlcCapabilities {
    pub ir_version: u32,
    pub core_ops: u64,
    pub composite_ops: u64,
    pub dtypes: u32,
    pub min_buffer_align: u32,
    pub max_scratchpad_bytes: u64,
    pub max_value_bytes: u64,
    pub head_dim_multiple_of: u32,
    pub matmul_k_multiple_of: u32,
    pub max_heads: u32,
    pub quant_formats: u32,
}

/// Opaque device handle.
#[repr(C)]
pub struct SlcDevice {
    _private: [u8; 0],
}

extern "C" {
    pub fn slc_device_create(ordinal: c_int, out: *mut *mut SlcDevice) -> c_int;
    pub fn slc_device_destroy(device: *mut SlcDevice);
    pub fn slc_last_error(device: *const SlcDevice, out: *mut SlcError) -> c_int;
    pub fn slc_get_capabilities(device: *const SlcDevice, out: *mut SlcCapabilities) -> c_int;
    pub fn slc_allocate_f32(device: *mut SlcDevice, elements: u64, align: u64, out: *mut u32) -> c_int;
    pub fn slc_allocate_u32(device: *mut SlcDevice, elements: u64, align: u64, out: *mut u32) -> c_int;
    pub fn slc_upload_f32(device: *mut SlcDevice, buffer: u32, data: *const f32, len: u64) -> c_int;
    pub fn slc_upload_u32(device: *mut SlcDevice, buffer: u32, data: *const u32, len: u64) -> c_int;
    pub fn slc_download_f32(device: *mut SlcDevice, buffer: u32, out: *mut f32, len: u64) -> c_int;
    pub fn slc_download_u32(device: *mut SlcDevice, buffer: u32, out: *mut u32, len: u64) -> c_int;
    pub fn slc_dispatch(
        device: *mut SlcDevice,
        op: *const SlcOp,
        inputs: *const SlcBufferRef,
        input_values: *const SlcValue,
        n_inputs: u64,
        outputs: *const SlcBufferRef,
        output_values: *const SlcValue,
        n_outputs: u64,
        scalars: *const u32,
        n_scalars: u64,
    ) -> c_int;
    pub fn slc_synchronize(device: *mut SlcDevice) -> c_int;
    pub fn slc_bind_quant(device: *mut SlcDevice, codes: u32, scales: u32, format: u32, group: u32) -> c_int;
    pub fn slc_set_capture(device: *mut SlcDevice, enabled: c_int) -> c_int;
    pub fn slc_comm_unique_id(out_id: *mut u8) -> c_int;
    pub fn slc_comm_init(device: *mut SlcDevice, unique_id: *const u8, rank: c_int, world: c_int) -> c_int;
    pub fn slc_comm_abort(device: *mut SlcDevice) -> c_int;
    pub fn slc_device_stream(device: *mut SlcDevice, out_stream: *mut *mut c_void) -> c_int;
}
