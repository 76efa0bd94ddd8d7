//! The CUDA branches of the model's `int8_kv_ops` module
//! (app/src/model/int8_kv_ops.rs:11-103) on libpp_b200, for candle-core
//! 0.11 with its CUDA backend (the app's vendored copy).
//!
//! The app keeps its functions and their host checks (`geometry`, the
//! `ensure!`s of int8_kv_ops.rs:42-53) and replaces each `#[cfg(feature =
//! "cuda")]` branch with a call into this module:
//!   quantize   -> [`quantize`]    (was cuda::Scale + cuda::Pack, int8_kv_ops.rs:23-27)
//!   dequantize -> [`dequantize`]  (was cuda::Pack{unpack}, :37-38)
//!   attention  -> [`attention`]   (was cuda::Attention, :49-52)
//!   prepare    -> [`prepare`]     (the on-device self-check, :57-103)
//! Each op reads the CudaStorage slices at their layout's start offset (as the
//! app's cuda_fwd does) and launches on the device's Candle stream.  Unlike
//! the app's split of 128, `split_tokens == 0` passes 0 to the library, which
//! balances tokens over the SMs and merges split rows inside the kernel.
use std::os::raw::c_void;

use candle_core::backend::BackendStorage;
use candle_core::cuda_backend::cudarc::driver::{DevicePtr, DevicePtrMut};
use candle_core::{CpuStorage, CudaStorage, CustomOp2, CustomOp3, DType, Device, Layout, Shape, Storage, Tensor};

use crate as sys;

fn wrap(e: sys::PpError) -> candle_core::Error {
    candle_core::Error::Msg(e.to_string())
}

fn cuda_only<T>() -> candle_core::Result<T> {
    candle_core::bail!("KV INT8 fused attention is only supported by the CUDA native provider")
}

/// quantize: packed u8 [h, n, d] is the op's output; the f32 scales [h, n]
/// are written into `scales`, a tensor the caller has just created for them.
struct Quantize {
    rows: usize,
    head_dim: usize,
}

impl CustomOp2 for Quantize {
    fn name(&self) -> &'static str {
        "pp-b200-quantize"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout) -> candle_core::Result<(CpuStorage, Shape)> {
        cuda_only()
    }

    fn cuda_fwd(&self, x: &CudaStorage, xl: &Layout, s: &CudaStorage, sl: &Layout)
                -> candle_core::Result<(CudaStorage, Shape)> {
        let d = &x.device;
        let stream = d.cuda_stream();
        let n = self.rows * self.head_dim;
        let mut packed = unsafe { d.alloc::<u8>(n) }?;
        let dtype = if x.dtype() == DType::BF16 { sys::PP_DTYPE_BF16 } else { sys::PP_DTYPE_F32 };
        let status = {
            let (xp, _gx) = match dtype {
                sys::PP_DTYPE_BF16 => x.as_cuda_slice::<half::bf16>()?.slice(xl.start_offset()..).device_ptr(&stream),
                _ => x.as_cuda_slice::<f32>()?.slice(xl.start_offset()..).device_ptr(&stream),
            };
            let (sp, _gs) = s.as_cuda_slice::<f32>()?.slice(sl.start_offset()..).device_ptr(&stream);
            let (pp, _gp) = packed.device_ptr_mut(&stream);
            unsafe {
                sys::pp_b200_quantize(xp as *const c_void, dtype, self.rows as u64, self.head_dim as u32,
                                      pp as *mut u8, sp as *mut f32, std::ptr::null_mut(),
                                      stream.cu_stream() as *mut c_void)
            }
        };
        sys::check(status).map_err(wrap)?;
        Ok((CudaStorage::wrap_cuda_slice(packed, d.clone()), xl.shape().clone()))
    }
}

/// int8_kv_ops::quantize, CUDA branch: (packed u8 [h, n, d], scales f32 [h, n]).
/// `input` is F32 or BF16 and contiguous (the app's `geometry` check).
pub fn quantize(input: &Tensor) -> candle_core::Result<(Tensor, Tensor)> {
    let (h, n, d) = input.dims3()?;
    let x = if matches!(input.dtype(), DType::F32 | DType::BF16) { input.clone() } else { input.to_dtype(DType::F32)? };
    let scales = Tensor::zeros((h, n), DType::F32, input.device())?;
    let packed = x.apply_op2_no_bwd(&scales, &Quantize { rows: h * n, head_dim: d })?;
    Ok((packed, scales))
}

struct Dequantize {
    rows: usize,
    head_dim: usize,
    dtype: DType,
}

impl CustomOp2 for Dequantize {
    fn name(&self) -> &'static str {
        "pp-b200-dequantize"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout) -> candle_core::Result<(CpuStorage, Shape)> {
        cuda_only()
    }

    fn cuda_fwd(&self, p: &CudaStorage, pl: &Layout, s: &CudaStorage, sl: &Layout)
                -> candle_core::Result<(CudaStorage, Shape)> {
        let d = &p.device;
        let stream = d.cuda_stream();
        let n = self.rows * self.head_dim;
        let bf16 = self.dtype == DType::BF16;
        let launch = |out: u64, pk: u64, sc: u64| unsafe {
            sys::pp_b200_dequantize(pk as *const u8, sc as *const f32, self.rows as u64, self.head_dim as u32,
                                    bf16 as i32, if bf16 { sys::PP_DTYPE_BF16 } else { sys::PP_DTYPE_F32 },
                                    out as *mut c_void, stream.cu_stream() as *mut c_void)
        };
        let (pk, _gp) = p.as_cuda_slice::<u8>()?.slice(pl.start_offset()..).device_ptr(&stream);
        let (sc, _gs) = s.as_cuda_slice::<f32>()?.slice(sl.start_offset()..).device_ptr(&stream);
        if bf16 {
            let mut out = unsafe { d.alloc::<half::bf16>(n) }?;
            let status = {
                let (op, _go) = out.device_ptr_mut(&stream);
                launch(op, pk, sc)
            };
            sys::check(status).map_err(wrap)?;
            Ok((CudaStorage::wrap_cuda_slice(out, d.clone()), pl.shape().clone()))
        } else {
            let mut out = unsafe { d.alloc::<f32>(n) }?;
            let status = {
                let (op, _go) = out.device_ptr_mut(&stream);
                launch(op, pk, sc)
            };
            sys::check(status).map_err(wrap)?;
            Ok((CudaStorage::wrap_cuda_slice(out, d.clone()), pl.shape().clone()))
        }
    }
}

/// int8_kv_ops::dequantize, CUDA branch: (i8) packed * scale as `dtype`;
/// BF16 is rounded once from the f32 product, as `.to_dtype(BF16)` does.
pub fn dequantize(packed: &Tensor, scale: &Tensor, dtype: DType) -> candle_core::Result<Tensor> {
    let (h, n, d) = packed.dims3()?;
    let direct = if dtype == DType::BF16 { DType::BF16 } else { DType::F32 };
    let out = packed.apply_op2_no_bwd(scale, &Dequantize { rows: h * n, head_dim: d, dtype: direct })?;
    if out.dtype() == dtype { Ok(out) } else { out.to_dtype(dtype) }
}

/// int8_kv_ops::attention, CUDA branch: reference mode (history of past[b]
/// int8 tokens plus the f32 scratch token), f32 [rows, 1, d] out.
struct Attention {
    ks: Tensor,
    vs: Tensor,
    sk: Tensor,
    sv: Tensor,
    past: Tensor,
    rows: usize,
    capacity: usize,
    heads: usize,
    head_dim: usize,
    split_tokens: usize,
}

impl CustomOp3 for Attention {
    fn name(&self) -> &'static str {
        "pp-b200-int8-attention"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout)
               -> candle_core::Result<(CpuStorage, Shape)> {
        cuda_only()
    }

    fn cuda_fwd(&self, q: &CudaStorage, ql: &Layout, k: &CudaStorage, kl: &Layout, v: &CudaStorage, vl: &Layout)
                -> candle_core::Result<(CudaStorage, Shape)> {
        let d = &q.device;
        let stream = d.cuda_stream();
        let (ks, ksl) = self.ks.storage_and_layout();
        let (vs, vsl) = self.vs.storage_and_layout();
        let (sk, skl) = self.sk.storage_and_layout();
        let (sv, svl) = self.sv.storage_and_layout();
        let (past, pl) = self.past.storage_and_layout();
        macro_rules! dev_ptr {
            ($storage:expr, $layout:expr, $ty:ty) => {
                match &*$storage {
                    Storage::Cuda(s) => s.as_cuda_slice::<$ty>()?.slice($layout.start_offset()..).device_ptr(&stream),
                    _ => candle_core::bail!("INT8 attention device mismatch"),
                }
            };
        }
        let (qp, _g0) = q.as_cuda_slice::<f32>()?.slice(ql.start_offset()..).device_ptr(&stream);
        let (kp, _g1) = k.as_cuda_slice::<u8>()?.slice(kl.start_offset()..).device_ptr(&stream);
        let (vp, _g2) = v.as_cuda_slice::<u8>()?.slice(vl.start_offset()..).device_ptr(&stream);
        let (ksp, _g3) = dev_ptr!(ks, ksl, f32);
        let (vsp, _g4) = dev_ptr!(vs, vsl, f32);
        let (skp, _g5) = dev_ptr!(sk, skl, f32);
        let (svp, _g6) = dev_ptr!(sv, svl, f32);
        let (lp, _g7) = dev_ptr!(past, pl, u32);
        let arena = sys::PpKvArena {
            struct_size: std::mem::size_of::<sys::PpKvArena>() as u32,
            rows: self.rows as u32,
            heads: self.heads as u32,
            head_dim: self.head_dim as u32,
            capacity: self.capacity as u32,
            reserved: 0,
            k: kp as *mut u8,
            v: vp as *mut u8,
            k_scale: ksp as *mut f32,
            v_scale: vsp as *mut f32,
        };
        let params = sys::PpAttnParams {
            split_tokens: if self.split_tokens == 0 { 0 } else { self.split_tokens.clamp(32, 1024) as u32 },
            ..Default::default()
        };
        // the workspace, like the app's partials, is allocated per call
        let ws_bytes = unsafe { sys::pp_b200_attention_workspace_size(&arena, &params) };
        if ws_bytes == 0 {
            candle_core::bail!("INT8 attention geometry differs: {}", sys::last_error());
        }
        let mut ws = unsafe { d.alloc::<u8>(ws_bytes) }?;
        let mut out = unsafe { d.alloc::<f32>(self.rows * self.head_dim) }?;
        let status = {
            let (wp, _gw) = ws.device_ptr_mut(&stream);
            let (op, _go) = out.device_ptr_mut(&stream);
            unsafe {
                sys::pp_b200_decode_attention(&arena, &params, qp as *const c_void, skp as *const f32,
                                              svp as *const f32, lp as *const u32, op as *mut c_void,
                                              wp as *mut c_void, ws_bytes, std::ptr::null_mut(),
                                              stream.cu_stream() as *mut c_void)
            }
        };
        sys::check(status).map_err(wrap)?;
        Ok((CudaStorage::wrap_cuda_slice(out, d.clone()), (self.rows, 1, self.head_dim).into()))
    }
}

/// int8_kv_ops::attention, CUDA branch (the app's checks have already run).
#[allow(clippy::too_many_arguments)]
pub fn attention(q: &Tensor, k: &Tensor, v: &Tensor, ks: &Tensor, vs: &Tensor, sk: &Tensor, sv: &Tensor,
                 past: &Tensor, heads: usize, split_tokens: usize) -> candle_core::Result<Tensor> {
    let (rows, capacity, head_dim) = k.dims3()?;
    q.apply_op3_no_bwd(k, v, &Attention {
        ks: ks.clone(),
        vs: vs.clone(),
        sk: sk.clone(),
        sv: sv.clone(),
        past: past.clone(),
        rows,
        capacity,
        heads,
        head_dim,
        split_tokens,
    })
}

/// int8_kv_ops::prepare: the library's on-device self-check with the app's
/// fixtures and tolerances.
pub fn prepare(device: &Device) -> candle_core::Result<()> {
    let ordinal = match device {
        Device::Cuda(d) => d.ordinal() as i32,
        _ => candle_core::bail!("KV INT8 needs CUDA in the native provider"),
    };
    sys::check(unsafe { sys::pp_b200_prepare(ordinal) }).map_err(wrap)
}
