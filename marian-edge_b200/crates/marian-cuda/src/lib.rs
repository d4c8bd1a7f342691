//! marian-cuda: marian-edge's Q8 greedy translation path on NVIDIA B200.
//!
//! The compute runs in libmarian_cuda.so (hand-written sm_100a kernels:
//! tcgen05 int8 GEMMs, packed varlen encoder attention, paged decode
//! attention, a device-side continuous batcher); this crate is the Rust host
//! side that marian-edge's server links:
//!
//! * [`CudaEngine`] is the token-id seam the CPU backend's engines fill
//!   (`CpuTokenEngine::translate_token_ids`, crates/marian-cpu/src/
//!   backend.rs:48-57; `Q8CpuEngine::translate_token_ids`, q8_engine.rs:353-466);
//! * [`CudaBackend`] implements `marian_core::TranslationBackend`
//!   (crates/marian-core/src/backend.rs:7-38) over text: long inputs split
//!   by `marian_core::segment_text`, SentencePiece encode + EOS, one output
//!   budget per input shared by its segments, decode, and the original
//!   separators re-inserted -- the rules of the CPU backend's adapter
//!   (crates/marian-cpu/src/backend.rs:107-346);
//! * [`start_cuda_translator`] is the server arm: one scheduler worker per
//!   GPU, each owning a full model replica (`Translator::start_pool`, the
//!   worker index picks the device).
//!
//! Like every marian-edge backend, a `CudaBackend` is created, used and
//! dropped on the scheduler's owner thread; it is neither `Send` nor `Sync`.
//!
//! Written against marian-edge v0.7.0's interfaces; not compiled on the
//! image it was written on (no Rust toolchain there).

mod ffi;

use std::ffi::CStr;
use std::marker::PhantomData;
use std::path::{Path, PathBuf};
use std::sync::Arc;

use marian_core::{
    BackendError, BackendInfo, SchedulerConfig, TranslationBackend, TranslationInput,
    TranslationOutput, Translator, segment_text,
};
use marian_model::ModelManifest;

/// marian-cpu/src/limits.rs:3 and :7.
const MAXIMUM_SOURCE_TOKENS: usize = 256;
const MAXIMUM_TRANSLATION_SEGMENTS: usize = 4096;
/// Generation steps per row (limits.rs:4): the output capacity per row.
const MAXIMUM_GENERATION_STEPS: usize = 256;

/// Engine options (the `mc_config` fields).
#[derive(Clone, Debug)]
pub struct CudaConfig {
    pub device: i32,
    pub max_inflight: u32,
    pub max_encode_tokens: u32,
    pub page_tokens: u32,
    pub lanes: u32,
}

impl Default for CudaConfig {
    fn default() -> Self {
        let mut raw = ffi::mc_config::default();
        unsafe { ffi::mc_config_default(&mut raw) };
        Self {
            device: raw.device,
            max_inflight: raw.max_inflight,
            max_encode_tokens: raw.max_encode_tokens,
            page_tokens: raw.page_tokens,
            lanes: raw.lanes,
        }
    }
}

impl CudaConfig {
    /// MARIAN_EDGE_CUDA_MAX_INFLIGHT, _PAGE_TOKENS and _LANES override the
    /// library defaults (1024, 16, 1).
    pub fn from_env(device: i32) -> Result<Self, BackendError> {
        let mut config = Self { device, ..Self::default() };
        let read = |name: &str, value: &mut u32| -> Result<(), BackendError> {
            if let Ok(text) = std::env::var(name) {
                *value = text
                    .parse()
                    .map_err(|_| BackendError::Model(format!("{name} must be an integer, got {text}")))?;
            }
            Ok(())
        };
        read("MARIAN_EDGE_CUDA_MAX_INFLIGHT", &mut config.max_inflight)?;
        read("MARIAN_EDGE_CUDA_PAGE_TOKENS", &mut config.page_tokens)?;
        read("MARIAN_EDGE_CUDA_LANES", &mut config.lanes)?;
        Ok(config)
    }
}

/// A device engine holding one model replica.  `!Send`: it belongs to the
/// thread that created it, as the C ABI requires.
pub struct CudaEngine {
    raw: *mut ffi::mc_engine,
    info: ffi::mc_model_info,
    _owner_thread: PhantomData<*mut ()>,
}

fn status_error(status: ffi::mc_status, raw: *const ffi::mc_engine) -> BackendError {
    let mut buf = [0 as std::os::raw::c_char; 1024];
    if !raw.is_null() {
        unsafe { ffi::mc_last_error(raw, buf.as_mut_ptr(), buf.len()) };
    }
    let message = unsafe { CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned();
    match status {
        ffi::MC_INVALID_INPUT => BackendError::InvalidInput(message),
        ffi::MC_MODEL => BackendError::Model(message),
        ffi::MC_DEVICE_TIMEOUT => BackendError::Inference(format!("device wait timed out: {message}")),
        ffi::MC_CUDA => BackendError::Inference(format!("CUDA failure: {message}")),
        _ => BackendError::Inference(message),
    }
}

fn check(status: ffi::mc_status, raw: *const ffi::mc_engine) -> Result<(), BackendError> {
    if status == ffi::MC_OK { Ok(()) } else { Err(status_error(status, raw)) }
}

impl CudaEngine {
    /// `Q8CpuEngine::from_bytes` (q8_engine.rs:175-184) on a GPU: parses the
    /// Marian binary v1 model, validates its Q8 schema and uploads it; the
    /// manifest's lexical shortlist, when given, restricts each sentence's
    /// candidates (shortlist.rs:150-198).
    pub fn load(
        weights: &[u8],
        shortlist: Option<&[u8]>,
        max_length_factor: usize,
        config: &CudaConfig,
    ) -> Result<Self, BackendError> {
        let mut raw_config = ffi::mc_config::default();
        unsafe { ffi::mc_config_default(&mut raw_config) };
        raw_config.device = config.device;
        raw_config.max_inflight = config.max_inflight;
        raw_config.max_encode_tokens = config.max_encode_tokens;
        raw_config.page_tokens = config.page_tokens;
        raw_config.lanes = config.lanes;
        raw_config.max_length_factor = u32::try_from(max_length_factor)
            .map_err(|_| BackendError::Model("max_length_factor does not fit u32".into()))?;
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::mc_create(&raw_config, &mut raw) }, std::ptr::null())?;
        let mut engine = Self { raw, info: ffi::mc_model_info::default(), _owner_thread: PhantomData };
        check(unsafe { ffi::mc_load_marian_bin(raw, weights.as_ptr(), weights.len()) }, raw)?;
        if let Some(bytes) = shortlist {
            check(unsafe { ffi::mc_load_shortlist(raw, bytes.as_ptr(), bytes.len()) }, raw)?;
        }
        check(unsafe { ffi::mc_model_info_get(raw, &mut engine.info) }, raw)?;
        Ok(engine)
    }

    pub fn is_ready(&self) -> bool {
        unsafe { ffi::mc_is_ready(self.raw) != 0 }
    }

    pub fn dim(&self) -> usize {
        self.info.dim as usize
    }

    /// Packed batch in, `(tokens, offsets)` out: offsets has batch + 1
    /// entries and each row holds its generated tokens (EOS included when
    /// generated), the contract of `BatchOutput` (engine.rs:82).
    pub fn translate_token_ids(
        &self,
        tokens: &[i32],
        offsets: &[u32],
        max_output_tokens: &[usize],
    ) -> Result<(Vec<i32>, Vec<u32>), BackendError> {
        let batch = offsets.len().saturating_sub(1);
        if max_output_tokens.len() != batch {
            return Err(BackendError::InvalidInput(format!(
                "{} output limits for {batch} packed sources",
                max_output_tokens.len()
            )));
        }
        let limits: Vec<u32> = max_output_tokens.iter().map(|&v| v.min(u32::MAX as usize) as u32).collect();
        let mut out = vec![0_i32; batch.max(1) * MAXIMUM_GENERATION_STEPS];
        let mut out_offsets = vec![0_u32; batch + 1];
        let batch_u32 = u32::try_from(batch).map_err(|_| BackendError::InvalidInput("batch exceeds u32".into()))?;
        check(
            unsafe {
                ffi::mc_translate_token_ids(
                    self.raw,
                    tokens.as_ptr(),
                    tokens.len(),
                    offsets.as_ptr(),
                    batch_u32,
                    limits.as_ptr(),
                    std::ptr::null(),
                    out.as_mut_ptr(),
                    out.len(),
                    out_offsets.as_mut_ptr(),
                )
            },
            self.raw,
        )?;
        out.truncate(out_offsets[batch] as usize);
        Ok((out, out_offsets))
    }
}

impl Drop for CudaEngine {
    fn drop(&mut self) {
        unsafe { ffi::mc_destroy(self.raw) };
    }
}

/// The text side of a backend: the tokenizer pair of the model directory.
pub trait PieceTokenizer {
    fn encode(&self, text: &str) -> Result<Vec<i32>, String>;
    fn decode(&self, ids: &[i32]) -> Result<String, String>;
    fn vocabulary_size(&self) -> usize;
}

impl PieceTokenizer for marian_tokenizer::Tokenizer {
    fn encode(&self, text: &str) -> Result<Vec<i32>, String> {
        marian_tokenizer::Tokenizer::encode(self, text).map_err(|e| e.to_string())
    }
    fn decode(&self, ids: &[i32]) -> Result<String, String> {
        marian_tokenizer::Tokenizer::decode(self, ids).map_err(|e| e.to_string())
    }
    fn vocabulary_size(&self) -> usize {
        self.len()
    }
}

/// `TranslationBackend` over a [`CudaEngine`].
pub struct CudaBackend {
    engine: CudaEngine,
    source: Arc<dyn PieceTokenizer>,
    target: Arc<dyn PieceTokenizer>,
    source_lang: String,
    target_lang: String,
    model_id: String,
    eos_id: i32,
    device: i32,
}

impl CudaBackend {
    /// Loads a checksum-verified `precision: "q8"` model directory onto one
    /// GPU (the files `Q8CpuBackend::load` reads, backend.rs:507-535).
    pub fn load(model_dir: impl AsRef<Path>, config: &CudaConfig) -> Result<Self, BackendError> {
        let model_dir = model_dir.as_ref();
        let manifest = ModelManifest::load(model_dir)?;
        manifest.verify_runtime_files(model_dir)?;
        if manifest.precision != "q8" {
            return Err(BackendError::Model(format!(
                "the CUDA backend runs precision q8 models, got {}",
                manifest.precision
            )));
        }
        let read = |name: &str| {
            std::fs::read(model_dir.join(name)).map_err(|error| {
                BackendError::Model(format!("failed to read {}: {error}", model_dir.join(name).display()))
            })
        };
        let weights = read(&manifest.weights)?;
        let shortlist = manifest.shortlist.as_deref().map(read).transpose()?;
        let open = |name: &str| {
            marian_tokenizer::Tokenizer::open(model_dir.join(name))
                .map_err(|error| BackendError::Model(format!("failed to load tokenizer {name}: {error}")))
        };
        let source = open(&manifest.source_vocab)?;
        let target = open(&manifest.target_vocab)?;
        let engine = CudaEngine::load(
            &weights,
            shortlist.as_deref(),
            manifest.architecture.max_length_factor,
            config,
        )?;
        Ok(Self {
            engine,
            source: Arc::new(source),
            target: Arc::new(target),
            source_lang: manifest.source_lang.clone(),
            target_lang: manifest.target_lang.clone(),
            model_id: manifest.model_id.clone(),
            eos_id: manifest.architecture.eos_id,
            device: config.device,
        })
    }
}

/// One input's segments while its translation is assembled.
struct Piece {
    text: Option<String>,
    separator: String,
    input_tokens: usize,
    output_tokens: usize,
}

impl TranslationBackend for CudaBackend {
    fn info(&self) -> BackendInfo {
        BackendInfo {
            name: "cuda".into(),
            device: format!("NVIDIA B200 (cuda:{})", self.device),
            model: self.model_id.clone(),
            precision: "q8".into(),
            attention: Some("varlen-encoder+paged-decode".into()),
            supports_batching: true,
        }
    }

    fn is_ready(&self) -> bool {
        self.engine.is_ready()
    }

    fn translate_batch(
        &mut self,
        inputs: &[TranslationInput],
    ) -> Result<Vec<TranslationOutput>, BackendError> {
        for input in inputs {
            if input.source_lang != self.source_lang || input.target_lang != self.target_lang {
                return Err(BackendError::UnsupportedDirection(format!(
                    "{} -> {}; loaded model is {} -> {}",
                    input.source_lang, input.target_lang, self.source_lang, self.target_lang
                )));
            }
        }
        // Plan: every input's segments, each non-empty one tokenized with EOS.
        let mut pieces: Vec<Vec<Piece>> = Vec::with_capacity(inputs.len());
        let mut queues: Vec<Vec<(usize, Vec<i32>)>> = Vec::with_capacity(inputs.len());
        let mut total = 0_usize;
        for input in inputs {
            let source = &self.source;
            let segments = segment_text(&input.text, MAXIMUM_SOURCE_TOKENS - 1, |text| {
                source.encode(text).map(|ids| ids.len())
            })
            .map_err(|error| BackendError::InvalidInput(error.to_string()))?;
            let mut planned = Vec::with_capacity(segments.len());
            let mut queue = Vec::new();
            for segment in segments {
                let content = segment.content(&input.text);
                let separator = segment.separator(&input.text).to_owned();
                if content.is_empty() {
                    planned.push(Piece { text: Some(String::new()), separator, input_tokens: 0, output_tokens: 0 });
                    continue;
                }
                total += 1;
                if total > MAXIMUM_TRANSLATION_SEGMENTS {
                    return Err(BackendError::InvalidInput(format!(
                        "batch requires more than {MAXIMUM_TRANSLATION_SEGMENTS} translated segments"
                    )));
                }
                let mut ids = self
                    .source
                    .encode(content)
                    .map_err(|e| BackendError::InvalidInput(format!("tokenizer encoding failed: {e}")))?;
                if ids.len() != segment.source_pieces {
                    return Err(BackendError::Inference(format!(
                        "source tokenizer returned {} pieces after sizing the segment as {}",
                        ids.len(),
                        segment.source_pieces
                    )));
                }
                let vocabulary = self.source.vocabulary_size();
                if let Some(&bad) = ids.iter().find(|&&t| t < 0 || t as usize >= vocabulary) {
                    return Err(BackendError::InvalidInput(format!(
                        "tokenizer returned source token {bad} outside vocabulary {vocabulary}"
                    )));
                }
                ids.push(self.eos_id);
                if ids.len() > MAXIMUM_SOURCE_TOKENS {
                    return Err(BackendError::Inference(format!(
                        "segmented source has {} tokens including EOS; maximum is {MAXIMUM_SOURCE_TOKENS}",
                        ids.len()
                    )));
                }
                queue.push((planned.len(), ids.clone()));
                planned.push(Piece { text: None, separator, input_tokens: ids.len(), output_tokens: 0 });
            }
            pieces.push(planned);
            queues.push(queue);
        }
        // Rounds: the next segment of every input with work and budget left
        // goes to the device in one packed batch (no CPU padding caps); an
        // input whose budget is spent gets empty text for the rest.
        let mut next = vec![0_usize; inputs.len()];
        let mut budget: Vec<usize> = inputs.iter().map(|i| i.max_output_tokens).collect();
        loop {
            let mut rows = Vec::new();
            for (i, queue) in queues.iter().enumerate() {
                while next[i] < queue.len() && budget[i] == 0 {
                    pieces[i][queue[next[i]].0].text = Some(String::new());
                    next[i] += 1;
                }
                if next[i] < queue.len() {
                    rows.push(i);
                }
            }
            if rows.is_empty() {
                break;
            }
            let mut tokens = Vec::new();
            let mut offsets = vec![0_u32];
            let mut limits = Vec::with_capacity(rows.len());
            for &i in &rows {
                tokens.extend_from_slice(&queues[i][next[i]].1);
                offsets.push(
                    u32::try_from(tokens.len())
                        .map_err(|_| BackendError::InvalidInput("packed source token count exceeds u32".into()))?,
                );
                limits.push(budget[i]);
            }
            let (out, out_offsets) = self.engine.translate_token_ids(&tokens, &offsets, &limits)?;
            for (row, &i) in rows.iter().enumerate() {
                let generated = &out[out_offsets[row] as usize..out_offsets[row + 1] as usize];
                budget[i] = budget[i].checked_sub(generated.len()).ok_or_else(|| {
                    BackendError::Inference("CUDA engine exceeded the max_output_tokens budget".into())
                })?;
                let ids: Vec<i32> = generated.iter().copied().filter(|&t| t != self.eos_id).collect();
                let text = self
                    .target
                    .decode(&ids)
                    .map_err(|e| BackendError::Inference(format!("tokenizer decoding failed: {e}")))?;
                let piece = &mut pieces[i][queues[i][next[i]].0];
                piece.text = Some(text);
                piece.output_tokens = ids.len();
                next[i] += 1;
            }
        }
        pieces
            .into_iter()
            .map(|planned| {
                let mut output = TranslationOutput { text: String::new(), score: None, input_tokens: 0, output_tokens: 0 };
                for piece in planned {
                    let text = piece
                        .text
                        .ok_or_else(|| BackendError::Inference("segment has no translation result".into()))?;
                    output.text.push_str(&text);
                    output.text.push_str(&piece.separator);
                    output.input_tokens += piece.input_tokens;
                    output.output_tokens += piece.output_tokens;
                }
                Ok(output)
            })
            .collect()
    }
}

/// The server's `BackendKind::Cuda` arm (crates/marian-server/src/main.rs:
/// 184-263 builds the other backends): one scheduler worker per listed GPU,
/// each loading a full model replica on its own device.
/// `MARIAN_EDGE_CUDA_DEVICES` (e.g. "0,1,2,3,4,5,6,7") lists the devices;
/// default: device 0 only.
pub fn start_cuda_translator(config: SchedulerConfig, model_dir: PathBuf) -> Result<Translator, BackendError> {
    let devices: Vec<i32> = match std::env::var("MARIAN_EDGE_CUDA_DEVICES") {
        Ok(list) => list
            .split(',')
            .map(|d| d.trim().parse::<i32>())
            .collect::<Result<_, _>>()
            .map_err(|_| BackendError::Model(format!("MARIAN_EDGE_CUDA_DEVICES is not a device list: {list}")))?,
        Err(_) => vec![0],
    };
    if devices.is_empty() {
        return Err(BackendError::Model("MARIAN_EDGE_CUDA_DEVICES lists no device".into()));
    }
    let count = devices.len();
    Translator::start_pool(config, count, move |worker| {
        let cuda = CudaConfig::from_env(devices[worker])?;
        CudaBackend::load(&model_dir, &cuda)
    })
}
