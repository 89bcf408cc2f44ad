// TensorFlow op definitions of the drop-in surface: `Sdpa` and `SdpaGrad`.
//
// Names, inputs, outputs, attrs (with defaults and order) and the type set are
// those of the reference (sdpa/sdpa_ops.cc:7-63), because `tf.load_op_library`
// users and their Python code (mha.py:8-29) bind to exactly these; the shape
// functions compute the same output shapes.
#include "tensorflow/core/framework/op.h"
#include "tensorflow/core/framework/shape_inference.h"

namespace tensorflow {
namespace {

using shape_inference::InferenceContext;
using shape_inference::ShapeHandle;

// output [B, S_q, D_v], stats [B, S_q]
Status SdpaShape(InferenceContext* c) {
  ShapeHandle q, k, v;
  TF_RETURN_IF_ERROR(c->WithRank(c->input(0), 3, &q));
  TF_RETURN_IF_ERROR(c->WithRank(c->input(1), 3, &k));
  TF_RETURN_IF_ERROR(c->WithRank(c->input(2), 3, &v));
  c->set_output(0, c->MakeShape({c->Dim(q, 0), c->Dim(q, 1), c->Dim(v, 2)}));
  c->set_output(1, c->MakeShape({c->Dim(q, 0), c->Dim(q, 1)}));
  return OkStatus();
}

// dq, dk, dv take the shapes of q, k, v
Status SdpaGradShape(InferenceContext* c) {
  for (int i = 0; i < 3; ++i) {
    ShapeHandle s;
    TF_RETURN_IF_ERROR(c->WithRank(c->input(i), 3, &s));
    c->set_output(i, s);
  }
  return OkStatus();
}

}  // namespace

REGISTER_OP("Sdpa")
    .Input("q: T")
    .Input("k: T")
    .Input("v: T")
    .Input("seed: uint64")
    .Input("offset: uint64")
    .Attr("scale: float = 1.0")
    .Attr("dropout: float = 0.0")
    .Attr("causal_mask: bool = false")
    .Attr("T: {half, float}")
    .Output("output: T")
    .Output("stats: float")
    .SetShapeFn(SdpaShape);

REGISTER_OP("SdpaGrad")
    .Input("q: T")
    .Input("k: T")
    .Input("v: T")
    .Input("out: T")
    .Input("stats: float")
    .Input("do: T")
    .Input("seed: uint64")
    .Input("offset: uint64")
    .Output("dq: T")
    .Output("dk: T")
    .Output("dv: T")
    .Attr("dropout: float = 0.0")
    .Attr("scale: float = 1.0")
    .Attr("causal_mask: bool = false")
    .Attr("T: {half, float}")
    .SetShapeFn(SdpaGradShape);

}  // namespace tensorflow
