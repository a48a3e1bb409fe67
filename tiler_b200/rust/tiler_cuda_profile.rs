// The tiler-cuda crate's target profile and payload metadata.
// Generated from tiler_b200/target_profile.py by
// `python -m tiler_b200.target_profile --rust`; regenerate, do not edit.

pub const PROFILE_KEY: &str = "tiler.cuda.sm_100a";
pub const PRODUCER: &str = "tiler-cuda";

fn guarantee(reference: &str) -> Result<TargetFactSource, TargetProfileBuildError> {
    let producer = TargetFactProducerIdentity::new(PRODUCER.to_owned(), 1)
        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;
    let reference = TargetNormativeReferenceIdentity::new(reference.to_owned(), 1)
        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;
    Ok(TargetFactSource::external_guarantee(producer, reference))
}

/// The sm_100a profile.  `cost_source` carries the measurement context of
/// the fold-step sweep (nvcc build, the B200 execution environment).
pub fn cuda_sm100a_profile(
    cost_source: Option<TargetCompileProfileMeasurementSource>,
) -> Result<TargetProfile, TargetProfileBuildError> {
    let key = TargetProfileKey::new(PROFILE_KEY.to_owned())
        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;
    let mut builder = TargetProfileBuilder::new(key);
    let ieee = guarantee("ieee.754.2019.binary32")?;
    let ptx = guarantee("nvidia.ptx-isa.sm_100a")?;

    // capability rows (tiler_cuda_device_facts_query)
    builder.declare_max_threads_per_grid_axis(2147483647, ptx.clone())?;
    builder.declare_max_threads_per_workgroup(1024, ptx.clone())?;
    builder.declare_max_buffer_bindings_per_entry(16, ptx.clone())?;
    builder.declare_index_arithmetic(IndexArithmeticSupport::CompleteU64, ptx.clone())?;
    builder.declare_device_address_width(DeviceAddressWidth::Bits64, ptx.clone())?;
    builder.declare_device_memory(true, ptx.clone())?;
    builder.declare_local_memory_bytes(232448, ptx.clone())?;

    // numerics rows: what every kernel does (IEEE binary32, one rounding per operator)
    let f32_subject = ScalarArithmetic::f32();
    builder.declare_input_subnormals(f32_subject.clone(), SubnormalMode::Preserve, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_input_subnormals(f32_subject.clone(), SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::PreservesSign }, ScalarSupport::Unsupported, ieee.clone())?;
    builder.declare_input_subnormals(f32_subject.clone(), SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::AlwaysPositive }, ScalarSupport::Unsupported, ieee.clone())?;
    builder.declare_result_subnormals(f32_subject.clone(), SubnormalMode::Preserve, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_result_subnormals(f32_subject.clone(), SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::PreservesSign }, ScalarSupport::Unsupported, ieee.clone())?;
    builder.declare_result_subnormals(f32_subject.clone(), SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::AlwaysPositive }, ScalarSupport::Unsupported, ieee.clone())?;
    builder.declare_contraction(f32_subject.clone(), NumericalPermission::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_contraction(f32_subject.clone(), NumericalPermission::Permitted, ScalarSupport::Unsupported, ieee.clone())?;
    builder.declare_reassociation(f32_subject.clone(), NumericalPermission::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    // permitted only as the grouping a provider proposal declares (the grid grouping)
    builder.declare_reassociation(f32_subject.clone(), NumericalPermission::Permitted, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_permutation(f32_subject.clone(), NumericalPermission::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_signed_zero(f32_subject.clone(), NumericalPermission::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_reciprocal_transform(f32_subject.clone(), NumericalPermission::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_approximate_intrinsics(f32_subject.clone(), ApproximationEnvelope::Forbidden, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_nan_assumptions(f32_subject.clone(), ExceptionalValueAssumption::MakeNoAssumption, ScalarSupport::Exact, ieee.clone())?;
    builder.declare_infinity_assumptions(f32_subject.clone(), ExceptionalValueAssumption::MakeNoAssumption, ScalarSupport::Exact, ieee.clone())?;

    // dtype dispatchability
    builder.declare_dtype_dispatchability(F32::resolved_type(), DTypeDispatchability::Dispatchable, ptx.clone())?;
    builder.declare_dtype_dispatchability(Bf16::resolved_type(), DTypeDispatchability::Dispatchable, ptx.clone())?;

    // the subgroup realization of the grouped fold's butterfly
    let subject = SubgroupRealizationSubject::new(
        SubgroupWidth::new(32).map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?,
        ArithmeticType::F32,
        SubgroupTransfer::InRangeXorShuffle,
    )
    .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;
    builder.declare_subgroup_realization(subject, SubgroupSupport::Realized, ptx.clone())?;

    // the measured cost row (a dispatch sweep on one B200; silence states no preference)
    if let Some(source) = cost_source {
        builder.declare_measured_saturated_parallel_fold_steps(10571, source)?;
    }
    builder.build()
}

/// PayloadMetadata for the sm_100a cubin (`code` = tiler_kernels.cubin).
pub fn cuda_payload_metadata(source_representation: RepresentationKey) -> PayloadMetadata {
    PayloadMetadata {
        source_representation,
        source: Vec::new(),
        provenance: PayloadProvenance {
            toolchain: "nvcc 12.9.86".to_owned(),
            target: "sm_100a".to_owned(),
            family: "tiler-cuda".to_owned(),
            language: "cuda-c++17".to_owned(),
            platform: PayloadPlatform::Unversioned,
            components: vec![
                ToolComponent { role: "cuda-compiler".to_owned(), version: "12.9.86".to_owned() },
            ],
            compile_flags: vec!["-std=c++17".to_owned(), "-O3".to_owned(), "-lineinfo".to_owned(), "-gencode".to_owned(), "arch=compute_100a,code=sm_100a".to_owned(), "-fmad=false".to_owned(), "-Xcompiler".to_owned(), "-fPIC".to_owned(), "-Xcompiler".to_owned(), "-Wall".to_owned(), "-Xptxas".to_owned(), "-v".to_owned()],
            link_flags: vec!["-Xlinker".to_owned(), "/usr/lib/x86_64-linux-gnu/libquadmath.so.0".to_owned()],
        },
        entries: vec![
            PayloadEntryMapping { entry_key: BackendEntryKey::new("sum_f32.grouped".to_owned()).expect("entry key"), symbol: "tiler_cuda.sum_f32.grouped".to_owned(), transports: Vec::new() },
            PayloadEntryMapping { entry_key: BackendEntryKey::new("max_f32.grouped".to_owned()).expect("entry key"), symbol: "tiler_cuda.max_f32.grouped".to_owned(), transports: Vec::new() },
            PayloadEntryMapping { entry_key: BackendEntryKey::new("rms_norm_f32".to_owned()).expect("entry key"), symbol: "tiler_cuda.rms_norm_f32".to_owned(), transports: Vec::new() },
            PayloadEntryMapping { entry_key: BackendEntryKey::new("rms_norm_bf16".to_owned()).expect("entry key"), symbol: "tiler_cuda.rms_norm_bf16".to_owned(), transports: Vec::new() },
            PayloadEntryMapping { entry_key: BackendEntryKey::new("rms_norm_quantize_i8".to_owned()).expect("entry key"), symbol: "tiler_cuda.rms_norm_quantize_i8".to_owned(), transports: Vec::new() },
        ],
        obligations: vec![PayloadTargetObligation { key: "subgroup-width".to_owned(), value: "32".to_owned() }],
    }
}
