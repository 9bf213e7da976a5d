//===----------------------------------------------------------------------===//
// --gawee-to-cuda: lower a gawee-dialect module to an LLVM-dialect module
// whose `_mlir_ciface_forward` runs the graph on a B200 through libgawee_cuda.
//
// Drop-in for middle/mlir/lib/Conversion/ of fwangdo/Gawee, registered in
// middle/mlir/tools/gawee-opt.cpp next to `--gawee-to-llvm` (a
// PassPipelineRegistration beside the one at gawee-opt.cpp:120-184).  It
// replaces the CPU pipeline of gawee-opt.cpp:120-184:
// instead of lowering every op to loops, the pass keeps the gawee-level
// `forward` as text in a global constant and emits
//
//   void _mlir_ciface_forward(MemRefDescriptor* result, MemRefDescriptor* arg0, ...)
//
// with the same signature the reference's LLVMRequestCWrappers produces
// (gawee-opt.cpp:171; consumed by back/gawee_aot.cpp:174-195), whose body
// packs the argument descriptor pointers into an array and calls
//
//   gawee_embedded_forward(text, device = 0, result, args, nargs)
//
// (include/gawee_cuda.h).  libgawee_cuda parses the text, plans it once per
// process and runs each call on the GPU.  The reference's `gawee-aot build`
// then links the module unchanged, with -lgawee_cuda added to its link line
// (gawee_aot.cpp:356-365).
//
// This file is source only in this repository: it needs the MLIR 22 headers
// and libraries that the reference's CMakeLists.txt:36 finds, which are not
// installed where this backend is built and tested.  The tested path to the
// same runtime is the C ABI (gawee_create / gawee_ciface_forward /
// gawee_embedded_forward) and the gawee-cuda-runner CLI.
//===----------------------------------------------------------------------===//

#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/Dialect/LLVMIR/LLVMDialect.h"
#include "mlir/IR/Builders.h"
#include "mlir/IR/BuiltinOps.h"
#include "mlir/Pass/Pass.h"
#include "llvm/Support/raw_ostream.h"

using namespace mlir;

namespace {

struct GaweeToCUDAPass : public PassWrapper<GaweeToCUDAPass, OperationPass<ModuleOp>> {
  StringRef getArgument() const override { return "gawee-to-cuda"; }
  StringRef getDescription() const override {
    return "Emit an LLVM-dialect module whose _mlir_ciface_forward runs the gawee graph with libgawee_cuda";
  }
  void getDependentDialects(DialectRegistry &registry) const override {
    registry.insert<LLVM::LLVMDialect>();
  }

  void runOnOperation() override {
    ModuleOp module = getOperation();
    auto forward = module.lookupSymbol<func::FuncOp>("forward");
    if (!forward) {
      module.emitError("gawee-to-cuda: no func.func @forward");
      return signalPassFailure();
    }
    if (forward.getNumResults() != 1) {
      forward.emitError("gawee-to-cuda: forward must return exactly one tensor (as gawee-aot requires)");
      return signalPassFailure();
    }
    const unsigned nargs = forward.getNumArguments();

    // 1. The gawee-level text libgawee_cuda plans, printed the way
    //    gawee-onnx-translate prints it: the default (custom) form.  gawee
    //    ops declare no assembly format, so they print in the generic form
    //    `"gawee.conv"(%0, %1) <{...}> : (...) -> ...`; func.func, return,
    //    arith.constant, tensor.empty, linalg.fill / generic / reduce print in
    //    their custom forms, with `#map = affine_map<...>` aliases at the top
    //    of the module.  That is the form the planner's parser reads
    //    (csrc/host/ir.cpp).  The full generic form (printGenericOpForm(true))
    //    would also print func.func and the module generically, which the
    //    parser does not accept, so it is not used.
    std::string text;
    {
      llvm::raw_string_ostream os(text);
      OpPrintingFlags flags;  // defaults: custom form where an op has one
      flags.elideLargeElementsAttrs(false);
      module.print(os, flags);
    }
    text.push_back('\0');

    // 2. Replace the module contents with the LLVM-dialect shim.
    MLIRContext *ctx = module.getContext();
    module.getBody()->clear();
    OpBuilder b = OpBuilder::atBlockEnd(module.getBody());
    Location loc = module.getLoc();
    auto ptr = LLVM::LLVMPointerType::get(ctx);
    auto i32 = b.getI32Type();
    auto i64 = b.getI64Type();
    auto voidTy = LLVM::LLVMVoidType::get(ctx);

    auto textTy = LLVM::LLVMArrayType::get(b.getI8Type(), text.size());
    LLVM::GlobalOp::create(b, loc, textTy, /*isConstant=*/true, LLVM::Linkage::Internal, "gawee_forward_text",
                           b.getStringAttr(text));

    auto calleeTy = LLVM::LLVMFunctionType::get(i32, {ptr, i32, ptr, ptr, i32});
    LLVM::LLVMFuncOp::create(b, loc, "gawee_embedded_forward", calleeTy);
    // Failure path: the reference's lowered code has no status, and its
    // launcher reports errors by exiting non-zero (back/gawee_aot.cpp:435-438),
    // so the shim prints gawee_last_error() and exits with status 1.
    LLVM::LLVMFuncOp::create(b, loc, "gawee_last_error", LLVM::LLVMFunctionType::get(i32, {ptr, ptr, i64}));
    LLVM::LLVMFuncOp::create(b, loc, "puts", LLVM::LLVMFunctionType::get(i32, {ptr}));
    LLVM::LLVMFuncOp::create(b, loc, "exit", LLVM::LLVMFunctionType::get(voidTy, {i32}));

    SmallVector<Type> params(nargs + 1, ptr);  // result descriptor, then one per argument
    auto shimTy = LLVM::LLVMFunctionType::get(voidTy, params);
    auto shim = LLVM::LLVMFuncOp::create(b, loc, "_mlir_ciface_forward", shimTy);
    Block *entry = shim.addEntryBlock(b);
    b.setInsertionPointToStart(entry);

    Value count = LLVM::ConstantOp::create(b, loc, i64, b.getI64IntegerAttr(nargs ? nargs : 1));
    Value array = LLVM::AllocaOp::create(b, loc, ptr, ptr, count, /*alignment=*/8);
    for (unsigned i = 0; i < nargs; ++i) {
      Value slot = LLVM::GEPOp::create(b, loc, ptr, ptr, array, ArrayRef<LLVM::GEPArg>{static_cast<int32_t>(i)});
      LLVM::StoreOp::create(b, loc, entry->getArgument(i + 1), slot);
    }
    Value textPtr = LLVM::AddressOfOp::create(b, loc, ptr, "gawee_forward_text");
    Value device = LLVM::ConstantOp::create(b, loc, i32, b.getI32IntegerAttr(0));
    Value n = LLVM::ConstantOp::create(b, loc, i32, b.getI32IntegerAttr(nargs));
    Value status = LLVM::CallOp::create(b, loc, TypeRange{i32}, "gawee_embedded_forward",
                                        ValueRange{textPtr, device, entry->getArgument(0), array, n})
                       .getResult();
    Value zero = LLVM::ConstantOp::create(b, loc, i32, b.getI32IntegerAttr(0));
    Value failed = LLVM::ICmpOp::create(b, loc, LLVM::ICmpPredicate::ne, status, zero);
    Block *okBlock = shim.addBlock();
    Block *failBlock = shim.addBlock();
    LLVM::CondBrOp::create(b, loc, failed, failBlock, okBlock);

    b.setInsertionPointToStart(failBlock);
    Value msgLen = LLVM::ConstantOp::create(b, loc, i64, b.getI64IntegerAttr(1024));
    Value msg = LLVM::AllocaOp::create(b, loc, ptr, b.getI8Type(), msgLen, /*alignment=*/1);
    Value null = LLVM::ZeroOp::create(b, loc, ptr);
    LLVM::CallOp::create(b, loc, TypeRange{i32}, "gawee_last_error", ValueRange{null, msg, msgLen});
    LLVM::CallOp::create(b, loc, TypeRange{i32}, "puts", ValueRange{msg});
    Value one = LLVM::ConstantOp::create(b, loc, i32, b.getI32IntegerAttr(1));
    LLVM::CallOp::create(b, loc, TypeRange{}, "exit", ValueRange{one});
    LLVM::UnreachableOp::create(b, loc);

    b.setInsertionPointToStart(okBlock);
    LLVM::ReturnOp::create(b, loc, ValueRange{});
  }
};

}  // namespace

namespace mlir::gawee {
std::unique_ptr<Pass> createGaweeToCUDAPass() { return std::make_unique<GaweeToCUDAPass>(); }
}  // namespace mlir::gawee
