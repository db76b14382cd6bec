//
//  QwenB200.swift -- the Swift host surface of the reference engine
//  (QwenEngine, QwenModel, QwenLayer, WeightLoader) over the B200 C ABI
//  (include/qwen_b200.h through include/module.modulemap).
//
//  Not built here: this machine and the GPU hosts have no swiftc.  A
//  maintainer adds this file next to the reference's QwenTokenizer.swift (the
//  tokenizer stays in Swift, QwenTokenizer.swift:11-71) and builds with
//      swiftc -I include -L qweninferenceengine_b200 -lqwen_b200 ...
//
//  Same public surface and error meaning as the reference:
//    QwenEngine(weightsPath:kernelsPath:)       InferenceEngine.swift:16-27
//    QwenEngine.generate(prompt:maxTokens:)     InferenceEngine.swift:29-52
//    QwenEngine.forward(tokenID:position:)      InferenceEngine.swift:54-271
//    QwenModel(weightsPath:)                    QwenModel.swift:22-34
//    QwenLayer(loader:index:)                   QwenLayer.swift:29-52 (file names)
//    WeightLoader / WeightLoadingError          WeightLoader.swift:11-52
//  The sampler, the KV cache and every kernel run on the GPU inside the
//  library; kernelsPath is accepted for source compatibility and unused (there
//  are no shaders to compile at run time).
//

import Foundation
import QwenB200

enum WeightLoadingError: Error {
    case fileNotFound(String)
    case bufferCreationFailed(String)
}

enum QwenB200Error: Error {
    case deviceUnavailable(String)   // MetalSetupError / fatalError sites of the reference
    case deviceTimeout(String)       // a bounded device wait gave up (the reference would hang)
    case invalidArgument(String)
    case failure(Int32, String)

    static func from(_ status: Int32) -> Error {
        let msg = String(cString: qwen_last_error())
        switch status {
        case QWEN_ERR_FILE_NOT_FOUND: return WeightLoadingError.fileNotFound(msg)
        case QWEN_ERR_BAD_WEIGHT_FILE: return WeightLoadingError.bufferCreationFailed(msg)
        case QWEN_ERR_NO_DEVICE: return QwenB200Error.deviceUnavailable(msg)
        case QWEN_ERR_DEVICE_TIMEOUT: return QwenB200Error.deviceTimeout(msg)
        case QWEN_ERR_INVALID_ARGUMENT: return QwenB200Error.invalidArgument(msg)
        default: return QwenB200Error.failure(status, msg)
        }
    }
}

@inline(__always) func check(_ status: Int32) throws {
    if status != QWEN_OK { throw QwenB200Error.from(status) }
}

/// WeightLoader.swift:16-52: the weight directory's file names and the
/// missing-file check; the bytes themselves are read by the library
/// (qwen_engine_load_weights), which reports a wrong size as bufferCreationFailed.
final class WeightLoader {
    let weightsDir: URL

    init(weightsDir: String) {
        self.weightsDir = URL(fileURLWithPath: weightsDir)
    }

    func path(relativePath: String) throws -> String {
        let fileURL = weightsDir.appendingPathComponent(relativePath)
        guard FileManager.default.fileExists(atPath: fileURL.path) else {
            throw WeightLoadingError.fileNotFound(fileURL.path)
        }
        return fileURL.path
    }

    func layerWeightPath(layer: Int, name: String) throws -> String {
        return try path(relativePath: "layer\(layer)/\(name).bin")
    }
}

/// QwenLayer.swift:29-52: the files one decoder layer is made of.
struct QwenLayer {
    static let fileNames = ["q_proj_4bit", "q_proj_scales", "k_proj_4bit", "k_proj_scales",
                            "v_proj_4bit", "v_proj_scales", "o_proj_4bit", "o_proj_scales",
                            "gate_proj_4bit", "gate_proj_scales", "up_proj_4bit", "up_proj_scales",
                            "down_proj_4bit", "down_proj_scales", "qkv_bias", "o_bias",
                            "mlp_down_bias"]
    let index: Int

    init(loader: WeightLoader, index: Int) throws {
        self.index = index
        _ = try loader.layerWeightPath(layer: index, name: "layer\(index)_norm")
        _ = try loader.layerWeightPath(layer: index, name: "layer\(index)_post_attn_norm")
        for name in QwenLayer.fileNames { _ = try loader.layerWeightPath(layer: index, name: name) }
    }
}

/// QwenModel.swift:11-35: checks the directory as the reference loads it
/// (global files, then 28 layers), so a missing file is reported with the
/// reference's error before the device is touched.
final class QwenModel {
    let loader: WeightLoader
    let weightsPath: String
    var layers: [QwenLayer] = []

    init(weightsPath: String, numLayers: Int = 28) throws {
        self.weightsPath = weightsPath
        self.loader = WeightLoader(weightsDir: weightsPath)
        _ = try loader.path(relativePath: "global/embed_tokens.bin")
        _ = try loader.path(relativePath: "global/final_norm.bin")
        for i in 0..<numLayers { layers.append(try QwenLayer(loader: loader, index: i)) }
    }
}

/// InferenceEngine.swift:9-369 on the B200 library.
final class QwenEngine {
    let model: QwenModel
    let tokenizer: QwenTokenizer
    private var handle: OpaquePointer?

    init(weightsPath: String, kernelsPath: String) async throws {
        self.model = try QwenModel(weightsPath: weightsPath)
        var cfg = qwen_engine_config()
        qwen_engine_config_default(&cfg)   // 1024 positions, T 0.7, top-p 0.8 (:273)
        var h: OpaquePointer?
        try check(qwen_engine_create(&cfg, &h))
        handle = h
        try check(qwen_engine_load_weights(handle, weightsPath))
        self.tokenizer = try await QwenTokenizer(weightsDir: weightsPath)
        print("QwenEngine Initialized and Ready.")
    }

    deinit { qwen_engine_destroy(handle) }

    /// generate(prompt:maxTokens:), InferenceEngine.swift:29-52: prefill, then
    /// print each token as it is produced until <|im_end|> / <|endoftext|>.
    func generate(prompt: String, maxTokens: Int = 64) throws {
        let tokens = tokenizer.encode(prompt: prompt)
        fflush(stdout)
        var currentToken = 0
        for i in 0..<tokens.count {
            currentToken = try forward(tokenID: tokens[i], position: i)
        }
        var currentPos = tokens.count
        for _ in 0..<maxTokens {
            if currentToken == 151645 || currentToken == 151643 { break }
            print(tokenizer.decode(tokens: [currentToken]), terminator: "")
            fflush(stdout)
            currentToken = try forward(tokenID: currentToken, position: currentPos)
            currentPos += 1
        }
        print("\n\n--- Generation Complete ---")
    }

    /// forward(tokenID:position:), InferenceEngine.swift:54-271: one decode
    /// step on the GPU, sampled there; returns the next token id.
    func forward(tokenID: Int, position: Int) throws -> Int {
        var next: Int32 = 0
        try check(qwen_engine_forward(handle, Int32(tokenID), Int32(position), &next))
        return Int(next)
    }

    /// The whole loop on token ids in one call (prefill on the tensor cores,
    /// decode steps without host round trips).
    func generate(tokens: [Int32], maxTokens: Int) throws -> [Int32] {
        var out = [Int32](repeating: 0, count: maxTokens)
        var n: Int32 = 0
        try check(qwen_engine_generate(handle, tokens, Int32(tokens.count), Int32(maxTokens), &out, &n))
        return Array(out.prefix(Int(n)))
    }
}
